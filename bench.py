"""bench.py -- KDA / MLA attention hot path on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|prefill|varlen|mla]
                    [--impl ours|reference]

Default workload (the headline): one KDA recurrent decode token for
B=256 sequences x H=32 heads, d_k=d_v=128, bf16 q/k/v/o, fp32 state [256,32,128,128]
resident in HBM (537 MB read and written per step, larger than L2, so no flush is needed
between steps). A step is one decode token for the whole batch. Metric: tokens/s.
Multi-GPU: every rank runs its own 256 sequences (weak scaling, no collective);
value = all ranks' tokens / max-over-ranks device time.

Other workloads (for the per-path records; one JSON line each):
  prefill  BASELINE config 2: T=32768, H=32, d=128, chunk 64 (tokens/s)
  varlen   BASELINE config 3: 16 sequences ~U[512,8192], H=64, heads sharded over the
           ranks, then the all-gather of the [sum T, 64*128] bf16 output (tokens/s)
  mla      BASELINE config 4: B=64, ctx 8192, 128 heads, latent 512 + rope 64 (tokens/s)
  mla_prefill  causal MLA prefill chunk over the latent cache: --tokens T (default 4096)
           new tokens of one sequence appended to the cache (kv_a_norm rows) and attended
           causally from position 0, 128 heads (tokens/s)
  moe_experts  one decode token through 16 routed experts' MXFP4 weights (k3_moe's expert
           step): w1 and w3 (3072 x 3584) on z, then w2 (3584 x 3072) on each expert's
           activation, as two batched launches (tokens/s)
  mla_layer  the whole MLA layer forward (k3_mla_cached) at the model's shape: hidden
           7168, 96 heads, q_lora 1536, latent 512 + rope 64, bf16 weights; --tokens T new
           tokens after --context positions already cached (default 1 after 8191)
  layer    the whole KDA layer forward (k3_kda_layer) at the model's shape: hidden 7168,
           96 heads of 128, conv 4, bf16 projection weights; --tokens T per call (default
           1: a decode step, weight streaming; e.g. 4096: a prefill chunk) (tokens/s)

--impl reference times the reference's own C implementation (oracle/_ref/libk3ref.so:
the unmodified k3_ops.c) on the host cores for the same workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "kimi-k3-in-c_b200"))

import workloads as W  # noqa: E402

# Algorithmic bytes per unit (one step of each workload): every tensor the step must read or
# write once, counted by the *_bytes functions below.
DECODE_B, DECODE_H, DECODE_D = 256, 32, 128


def decode_bytes(B, H, d):
    state = 2 * B * H * d * d * 4            # fp32 state read + written
    qkv = 3 * B * H * d * 2                  # bf16 q, k, v
    gate = B * H * d * 4 + B * H * 4         # fp32 g and beta
    out = B * H * d * 2                      # bf16 o
    return state + qkv + gate + out


def prefill_bytes(T, H, d, eb=2):
    """q, k, v in and o out at `eb` bytes per element, fp32 g and beta."""
    return 4 * T * H * d * eb + T * H * d * 4 + T * H * 4


def mla_bytes(B, ctx, H):
    return (B * ctx * 512 * 2 + B * ctx * 64 * 2 + 2 * H * 128 * 512 * 2 + B * H * 192 * 2
            + B * H * 128 * 2)


def mla_flops(B, ctx, H):
    return 2 * B * H * (128 * 512 + ctx * 576 + ctx * 512 + 512 * 128)


LAYER_E, LAYER_H, LAYER_D, LAYER_K = 7168, 96, 128, 4


def layer_weight_bytes(E, H, D):
    P = H * D
    return 2 * (4 * P * E + H * E + D * E + P * D + E * P)   # bf16 q,k,v,g,b,f_a,f_b,o


def layer_bytes(T, E, H, D, K):
    """HBM bytes one layer call must move at least: every weight once, the recurrent and
    conv state read and written, x in and out (activations between steps excluded)."""
    P = H * D
    return (layer_weight_bytes(E, H, D) + 2 * (H * D * D + 3 * P * (K - 1)) * 4
            + 2 * T * E * 4)


def layer_flops(T, E, H, D):
    """Projection FLOPs of one call (the recurrence adds < 3% at T = 4096)."""
    P = H * D
    return 2 * T * (4 * P * E + H * E + D * E + D * P + P * E)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self):
        return time.time()

    def stop(self, t0, t1):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [ln for (ts, ln) in self.lines if t0 - 0.15 <= ts <= t1 + 0.15] or \
            [ln for (_, ln) in self.lines]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in rows:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------- distributed
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
            self.dist = dist

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def allgather_obj(self, x):
        if self.world == 1:
            return [x]
        out = [None] * self.world
        self.dist.all_gather_object(out, x)
        return out

    def bcast_bytes(self, b: bytes | None) -> bytes:
        if self.world == 1:
            return b
        obj = [b]
        self.dist.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


# ---------------------------------------------------------------- cpu baseline
def cpu_decode_baseline(B, H, d, budget_s=6.0):
    """The reference's k3_kda_step (oracle/_ref, unmodified k3_ops.c) over the config-1
    batch on all host cores, repeated for about budget_s seconds."""
    from oracle import oracle
    if not oracle.ref_available():
        return None
    c = W.kda_config1(B=B, H=H, d=d)
    nth = oracle.ref().k3ref_max_threads()
    S = c["state"].copy()
    oracle.kda_decode(S[:1], c["q"][:1], c["k"][:1], c["v"][:1], c["g"][:1], c["beta"][:1],
                      use_ref=True, nthreads=nth)
    steps, t0 = 0, time.perf_counter()
    while True:
        _, S = oracle.kda_decode(S, c["q"], c["k"], c["v"], c["g"], c["beta"], use_ref=True,
                                 nthreads=nth)
        steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"value": B * steps / el, "unit": "tokens/s", "cores": nth, "kind": "reference",
            "sample": f"{steps} full config-1 decode steps (B={B}, H={H}, d={d}) through the "
                      f"reference k3_kda_step, OpenMP over the {B * H} (sequence, head) streams"}


# ----------------------------------------------------------------------- decode
def decode_config(B, H, d):
    """The config-1 workload description, identical in both arms."""
    return {"workload": "kda_decode_config1", "batch_per_gpu": B, "heads": H, "d_k": d,
            "d_v": d, "io": "bf16 q/k/v/o, fp32 g/beta/state",
            "parallelism": "sequence-shard (no collective)",
            "l2": "inputs larger than L2 (537 MB fp32 state per GPU)"}


def bench_decode(args, D: Dist):
    import k3cuda
    ctx = k3cuda.Context(D.local)
    B, H, d = DECODE_B, DECODE_H, DECODE_D
    c = W.kda_config1(seed=D.rank, B=B, H=H, d=d)
    qs = 1.0 / np.sqrt(np.float32(d))
    bf = W.f32_to_bf16
    dS = ctx.upload(c["state"])
    dq, dk, dv = ctx.upload(bf(c["q"])), ctx.upload(bf(c["k"])), ctx.upload(bf(c["v"]))
    dg, db = ctx.upload(c["g"]), ctx.upload(c["beta"])
    do = ctx.empty((B, H, d), np.uint16)

    def step():
        ctx.kda_decode(dS, do, dq, dk, dv, dg, db, B, H, d, d, qs)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    clk = ClockSampler(D.local)
    clk.start()
    time.sleep(0.3)
    D.barrier()
    ctx.sync()
    l0 = ctx.launches()
    t0 = clk.mark()
    ctx.record(0)
    for _ in range(args.steps):
        step()
    ctx.record(1)
    ctx.sync()
    t1 = clk.mark()
    D.barrier()
    l1 = ctx.launches()
    ms = ctx.elapsed_ms(0, 1)
    ms_max = D.max(ms)
    clocks = clk.stop(t0, t1)

    # e2e: the host-buffer entry point (k3cuda_kda_decode_host): q, k, v, g, beta from
    # page-locked host memory in and o back every step, the copies pipelined over batch
    # slices against the kernel
    hq, hk, hv = (ctx.pinned((B, H, d), np.uint16) for _ in range(3))
    hg = ctx.pinned((B, H, d), np.float32)
    hb = ctx.pinned((B, H), np.float32)
    ho = ctx.pinned((B, H, d), np.uint16)
    hq[...], hk[...], hv[...], hg[...], hb[...] = bf(c["q"]), bf(c["k"]), bf(c["v"]), c["g"], c["beta"]
    bi = sum(h.nbytes for h in (hq, hk, hv, hg, hb))
    bo = ho.nbytes
    nst = ctx.kda_decode_host_workspace(B, H, d, d)
    stage = ctx.empty((nst,), np.uint8)

    def e2e_step():
        ctx.kda_decode_host(dS, ho, hq, hk, hv, hg, hb, B, H, d, d, qs, stage, nst)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    ctx.sync()
    D.barrier()
    ctx.record(2)
    for _ in range(args.steps):
        e2e_step()
    ctx.record(3)
    ctx.sync()
    D.barrier()
    ms_e2e = D.max(ctx.elapsed_ms(2, 3))

    hbm, tf, src = peaks()
    per_launch_s = ms_max / 1e3 / args.steps
    alg = decode_bytes(B, H, d)
    achieved = alg / per_launch_s / 1e9
    toks = B * args.steps * D.world
    line = {
        "metric": "KDA recurrent decode tokens/s (BASELINE config 1: B=256, H=32, d=128)",
        "value": toks / (ms_max / 1e3), "unit": "tokens/s", "n_gpus": D.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "mixed",
        "data": "synthetic (seeded numpy: BASELINE config-1 distributions)",
        "config": decode_config(B, H, d),
        "e2e": {"value": toks / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": bi,
                "d2h_bytes_per_step": bo,
                "path": "k3cuda_kda_decode_host: page-locked host tensors, input copies "
                        "pipelined against the kernel over batch slices, output written to the "
                        "host by the kernel"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_source": src,
                     "traffic": None,
                     "algorithmic_bytes_per_launch": alg},
        "gpu_launches": int(l1 - l0),
        "clocks": clocks,
    }
    ctx.close()
    return line


# ------------------------------------------------------------------ timing helpers
def timed(ctx, D: Dist, step, steps, warmup, slots=(0, 1)):
    """W untimed steps, then K steps between CUDA events on the context's stream, bracketed by
    barrier + synchronize; returns (max-over-ranks ms, kernels launched, clocks)."""
    for _ in range(warmup):
        step()
    ctx.sync()
    clk = ClockSampler(D.local)
    clk.start()
    time.sleep(0.3)
    D.barrier()
    ctx.sync()
    l0 = ctx.launches()
    t0 = clk.mark()
    ctx.record(slots[0])
    for _ in range(steps):
        step()
    ctx.record(slots[1])
    ctx.sync()
    t1 = clk.mark()
    D.barrier()
    l1 = ctx.launches()
    ms = D.max(ctx.elapsed_ms(*slots))
    return ms, int(l1 - l0), clk.stop(t0, t1)


def timed_e2e(ctx, D: Dist, step, steps, warmup):
    """Same bracket without the clock sampler, for the host-buffer (end-to-end) leg."""
    for _ in range(max(1, warmup)):
        step()
    ctx.sync()
    D.barrier()
    ctx.record(2)
    for _ in range(steps):
        step()
    ctx.record(3)
    ctx.sync()
    D.barrier()
    return D.max(ctx.elapsed_ms(2, 3))


# ---------------------------------------------------------------------- prefill
PREFILL = {"cfg2": dict(H=32, name="kda_prefill_config2"),
           "cfg3": dict(H=64, name="kda_prefill_config3")}


def prefill_inputs(which, heads=None, tokens=None):
    if which == "cfg2":
        return W.kda_config2(T=tokens, heads=heads) if tokens else W.kda_config2(heads=heads)
    return W.kda_config3(heads=heads)


def prefill_sample(which, n=1024):
    """The first n tokens of config 2 or 3 at all heads, for the CPU baseline's sample (the
    reference's time per token and head does not depend on the values)."""
    H = PREFILL[which]["H"]
    t = W.kda_tokens_by_head(0 if which == "cfg2" else 1, n, H, 128, 128, True)
    t["cu_seqlens"] = np.array([0, n], np.int32)
    return t


def cpu_prefill_baseline(c, H, budget_s=5.0, tokens=1024):
    """The reference's own k3_kda_step (oracle/_ref) driven as its k3_kda_layer recurrence
    (k3_ops.c:908-938) over the first `tokens` tokens of the packed batch, all H heads,
    OpenMP over heads on every host core, repeated for about budget_s seconds."""
    from oracle import oracle
    if not oracle.ref_available():
        return None
    nth = oracle.ref().k3ref_max_threads()
    n = min(tokens, int(c["cu_seqlens"][-1]))
    sub = {x: np.ascontiguousarray(c[x][:n]) for x in ("q", "k", "v", "g", "beta")}
    cu = np.array([0, n], np.int32)
    calls, t0 = 0, time.perf_counter()
    while True:
        oracle.kda_recurrence(sub["q"], sub["k"], sub["v"], sub["g"], sub["beta"], cu,
                              use_ref=True, nthreads=nth)
        calls += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"value": n * calls / el, "unit": "tokens/s", "cores": nth, "kind": "reference",
            "sample": f"{calls} passes over the first {n} tokens x {H} heads (d=128) through "
                      f"the reference k3_kda_step, OpenMP over heads"}


def prefill_record(args, D: Dist, which, tokens=None, cpu=True):
    """BASELINE config 2 or 3. One rank: the whole batch. N ranks: heads split evenly, each
    rank's prefill writing its heads straight into every rank's full [T][H][d] output over
    NVLink (k3cuda_kda_prefill_gathered); timed both with the exchange and compute-only."""
    import k3cuda
    import sharding
    cfg = PREFILL[which]
    H_total, d = cfg["H"], 128
    R = D.world
    hs = sharding.head_shard(H_total, R, D.rank)
    Hl = hs.stop - hs.start
    c = prefill_inputs(which, heads=hs, tokens=tokens)
    cu = c["cu_seqlens"]
    T, nseq = int(cu[-1]), len(cu) - 1
    ctx = k3cuda.Context(D.local)
    f32 = getattr(args, "io", "bf16") == "f32"  # fp32 q/k/v/o: the path the C99 drop-ins take
    if f32 and R > 1:
        raise ValueError("--io f32 runs on one GPU (the gathered exchange is bf16)")
    et = np.float32 if f32 else np.uint16
    cv = (lambda a: a) if f32 else W.f32_to_bf16
    hq, hk, hv = (ctx.pinned((T, Hl, d), et) for _ in range(3))
    hg = ctx.pinned((T, Hl, d), np.float32)
    hb = ctx.pinned((T, Hl), np.float32)
    hq[...], hk[...], hv[...], hg[...], hb[...] = cv(c["q"]), cv(c["k"]), cv(c["v"]), c["g"], c["beta"]
    cpu_c = c if (cpu and R == 1 and D.rank == 0 and not args.no_cpu_baseline) else None
    del c
    dq, dk, dv = (ctx.empty((T, Hl, d), et) for _ in range(3))
    dg, db = ctx.empty((T, Hl, d), np.float32), ctx.empty((T, Hl), np.float32)
    h2d = [(dq, hq), (dk, hk), (dv, hv), (dg, hg), (db, hb)]
    L = k3cuda.lib()
    for dbuf, h in h2d:
        k3cuda.check(L.k3cuda_memcpy_h2d(ctx.h, dbuf.ptr, h.ctypes.data, h.nbytes))
    dS = ctx.empty((nseq, Hl, d, d), np.float32)
    dloc = ctx.empty((T, Hl, d), et)
    nws = ctx.kda_prefill_workspace(cu, Hl, d, d)
    ws = ctx.empty((nws,), np.uint8)
    qs = 1.0 / np.sqrt(np.float32(d))
    gather = R > 1
    if gather:
        uid = D.bcast_bytes(k3cuda.comm_unique_id() if D.rank == 0 else None)
        ctx.comm_init(R, D.rank, uid)
        dfull = ctx.empty((T, H_total, d), np.uint16)
        ctx.comm_register_full(dfull)

    io = k3cuda.F32 if f32 else k3cuda.BF16

    def step_local():
        dS.zero()
        ctx.kda_prefill(dS, dloc, dq, dk, dv, dg, db, cu, Hl, d, d, qs, ws, nws, io_dtype=io)

    def step_gather():
        dS.zero()
        ctx.kda_prefill_gathered(dS, dq, dk, dv, dg, db, cu, Hl, d, d, qs, ws, nws)

    step = step_gather if gather else step_local
    ms, launches, clocks = timed(ctx, D, step, args.steps, args.warmup)
    ms_compute = timed(ctx, D, step_local, args.steps, args.warmup)[0] if gather else ms

    check = None
    if gather:
        # (1) this rank's heads in its gathered buffer equal an unsharded run of the same heads
        # on this GPU; (2) every rank's gathered buffer holds the same bytes. Together: every
        # rank holds every rank's heads, bit for bit as computed by their owners.
        full = dfull.numpy()
        step_local()
        own = dloc.numpy()
        ok_own = bool(np.array_equal(full[:, hs], own))
        import hashlib
        digest = hashlib.blake2b(full.tobytes(), digest_size=16).hexdigest()
        digests = D.allgather_obj(digest)
        ok_same = len(set(digests)) == 1
        check = {"result": "pass" if (ok_own and ok_same) else "fail",
                 "own_heads_equal_unsharded": ok_own, "all_ranks_same_output": ok_same,
                 "what": "gathered [sum T, H, 128] output on every rank: its own heads vs an "
                         "unsharded prefill of them, and a blake2b digest compared across "
                         "ranks"}
        del full

    # e2e: this rank's inputs from page-locked host memory in, and the output back (with the
    # exchange, each rank reads back its 1/R share of the gathered rows, all heads)
    if gather:
        r0, r1 = D.rank * T // R, (D.rank + 1) * T // R
        row_bytes = H_total * d * 2
        src_ptr, nb = dfull.ptr + r0 * row_bytes, (r1 - r0) * row_bytes
    else:
        src_ptr, nb = dloc.ptr, dloc.nbytes
    ho = ctx.pinned((max(nb, 2) // 2,), np.uint16)

    def e2e_step():
        for dbuf, h in h2d:
            k3cuda.check(L.k3cuda_memcpy_h2d(ctx.h, dbuf.ptr, h.ctypes.data, h.nbytes))
        step()
        k3cuda.check(L.k3cuda_memcpy_d2h(ctx.h, ho.ctypes.data, src_ptr, nb))

    ms_e2e = timed_e2e(ctx, D, e2e_step, args.steps, args.warmup)
    hbm, tf, src = peaks()
    per = ms_compute / 1e3 / args.steps
    # fp32 q, k, v and o move twice the bytes of bf16 ones
    alg = prefill_bytes(T, Hl, d, 4 if f32 else 2)
    name = cfg["name"] if not tokens else f"kda_prefill_T{T}_reduced"
    if f32:
        name += "_fp32io"
    rec = {
        "metric": f"KDA chunked prefill tokens/s ({name})",
        "value": T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": R,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "ms_per_step_compute_only": ms_compute / args.steps,
        "value_compute_only": T * args.steps / (ms_compute / 1e3),
        "higher_is_better": True, "scaling": "strong", "dtype": "mixed",
        "config": {"workload": name, "tokens": T, "sequences": nseq, "heads_total": H_total,
                   "heads_per_gpu": Hl, "d": d, "chunk": 64,
                   "io": ("fp32 q/k/v/o/g/beta/state (fp32 intra-chunk kernel, tcgen05 "
                          "scan on bf16 hi/lo operands)" if f32 else
                          "bf16 q/k/v/o, fp32 g/beta/state"),
                   "parallelism": f"head-shard x{R}" + (", output exchange fused into the "
                                                        "prefill (peer stores over NVLink)"
                                                        if gather else ""),
                   "l2": "inputs larger than L2"},
        "e2e": {"value": T * args.steps / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(sum(h.nbytes for _, h in h2d)),
                "d2h_bytes_per_step": int(nb)},
        "roofline": {"bound": "hbm", "achieved": alg / per / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": alg / per / 1e9 / hbm, "peak_source": src, "traffic": None,
                     "algorithmic_bytes_per_launch": alg,
                     "basis": "compute-only time of this rank's heads"},
        "gpu_launches": launches, "clocks": clocks,
    }
    if check:
        rec["check"] = check
    if gather:
        # the exchange: every rank receives the other ranks' heads of the whole output; its
        # floor is those bytes over one GPU's NVLink ingress (the measured 770 GB/s peer copy)
        recv = (R - 1) * T * Hl * d * 2
        t_x = max(ms - ms_compute, 1e-6) / 1e3 / args.steps
        rec["exchange"] = {"bytes_received_per_gpu": recv, "ms_per_step": t_x * 1e3,
                           "achieved_gbs": recv / t_x / 1e9, "peak_gbs": 770.0,
                           "frac": recv / t_x / 1e9 / 770.0,
                           "floor_ms": recv / 770e9 * 1e3,
                           "basis": "time with the exchange minus compute-only time; peak = "
                                    "measured NVLink peer copy per direction per GPU"}
    ctx.close()
    if cpu_c is not None:
        rec["cpu_baseline"] = cpu_prefill_baseline(cpu_c, H_total)
    return rec


# -------------------------------------------------------------------------- mla
def cpu_mla_baseline(c, budget_s=5.0, nb=2):
    """The absorbed restatement of the reference's decode attention loop (k3_ops.c:381-411,
    oracle/k3_oracle.c orc_mla_absorbed_decode: fp64 dots and sum, expf) over `nb` of the
    config-4 sequences, all 128 heads, OpenMP over (sequence, head), for about budget_s s."""
    from oracle import oracle
    f = W.bf16_to_f32
    args_ = [np.ascontiguousarray(f(c[x][:nb])) for x in ("q_nope", "q_rope", "latent", "rope")]
    args_ += [f(c["w_uk"]), f(c["w_uv"])]
    lens = np.ascontiguousarray(c["ctx_lens"][:nb])
    nth = oracle.max_threads()
    calls, t0 = 0, time.perf_counter()
    while True:
        oracle.mla_absorbed_decode(*args_, lens, c["scale"], nthreads=nth)
        calls += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"value": nb * calls / el, "unit": "tokens/s", "cores": nth, "kind": "port",
            "sample": f"{calls} passes over {nb} of the 64 sequences (8192 positions, 128 heads) "
                      f"through the C restatement of the reference's attention loop"}


def mla_record(args, D: Dist, cpu=True):
    """64 sequences split evenly over the ranks (no collective)."""
    import k3cuda
    R = D.world
    B_all, ctxlen, H = 64, 8192, 128
    B = B_all // R
    if getattr(args, "batch", None):  # a rank's share of a larger job, for profiling
        B = args.batch
        B_all = B * R
    c = W.mla_config4(seed=D.rank, B=B, ctx=ctxlen, H=H)
    ctx = k3cuda.Context(D.local)
    d = [ctx.upload(c[x]) for x in ("q_nope", "q_rope", "latent", "rope", "w_uk", "w_uv")]
    out = ctx.empty((B, H, 128), np.uint16)
    nws = ctx.mla_decode_workspace(c["ctx_lens"], H)
    ws = ctx.empty((nws,), np.uint8)

    def step():
        ctx.mla_decode(out, *d, c["ctx_lens"], ctxlen, H, c["scale"], ws, nws,
                       out_dtype=k3cuda.BF16)

    ms, launches, clocks = timed(ctx, D, step, args.steps, args.warmup)
    # e2e: the step's queries in from page-locked memory, the output back (the latent cache
    # is resident device state, like the KDA recurrent state)
    hqn, hqr = ctx.pinned(c["q_nope"].shape, np.uint16), ctx.pinned(c["q_rope"].shape, np.uint16)
    hqn[...], hqr[...] = c["q_nope"], c["q_rope"]
    ho = ctx.pinned((B, H, 128), np.uint16)
    L = k3cuda.lib()

    def e2e_step():
        k3cuda.check(L.k3cuda_memcpy_h2d(ctx.h, d[0].ptr, hqn.ctypes.data, hqn.nbytes))
        k3cuda.check(L.k3cuda_memcpy_h2d(ctx.h, d[1].ptr, hqr.ctypes.data, hqr.nbytes))
        step()
        k3cuda.check(L.k3cuda_memcpy_d2h(ctx.h, ho.ctypes.data, out.ptr, ho.nbytes))

    ms_e2e = timed_e2e(ctx, D, e2e_step, args.steps, args.warmup)
    hbm, tf, src = peaks()
    per = ms / 1e3 / args.steps
    alg = mla_bytes(B, ctxlen, H)
    rec = {
        "metric": "MLA absorbed decode tokens/s (BASELINE config 4)",
        "value": B_all * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": R,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "strong", "dtype": "mixed",
        "config": {"workload": "mla_decode_config4", "batch": B_all, "batch_per_gpu": B,
                   "ctx": ctxlen, "heads": H, "io": "bf16 q/cache/W_UK/W_UV/out, fp32 softmax",
                   "parallelism": f"batch-shard x{R} (no collective)",
                   "l2": "inputs larger than L2 (latent+rope cache)"},
        "e2e": {"value": B_all * args.steps / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(hqn.nbytes + hqr.nbytes),
                "d2h_bytes_per_step": int(ho.nbytes)},
        "roofline": {"bound": "hbm", "achieved": alg / per / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": alg / per / 1e9 / hbm, "peak_source": src, "traffic": None,
                     "algorithmic_bytes_per_launch": alg,
                     "tensor_tflops": mla_flops(B, ctxlen, H) / per / 1e12},
        "gpu_launches": launches, "clocks": clocks,
    }
    ctx.close()
    if cpu and R == 1 and D.rank == 0 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = cpu_mla_baseline(c)
    return rec


def guarded(fn, *a, **kw):
    """A sub-record that failed on this rank is reported, not raised: the headline line still
    prints. (Every rank runs the same steps, so a failure in a collective ends on every rank
    under the communicator's deadline.)"""
    try:
        return fn(*a, **kw)
    except Exception as e:  # noqa: BLE001
        return {"error": f"{type(e).__name__}: {e}"}


# ------------------------------------------------------------------------ layer
def layer_inputs(seed, T, E=LAYER_E, H=LAYER_H, D=LAYER_D, K=LAYER_K):
    rng = np.random.default_rng(seed)
    w = W.kda_layer_weights(rng, E, H, D, K, pool=1 << 22, bf16=True)
    x = rng.standard_normal((T, E)).astype(np.float32)
    state = (0.05 * rng.standard_normal(H * D * D + 3 * H * D * (K - 1))).astype(np.float32)
    return w, x, state


def bench_layer(args, D: Dist):
    import k3cuda
    ctx = k3cuda.Context(D.local)
    E, H, Dh, K = LAYER_E, LAYER_H, LAYER_D, LAYER_K
    T = args.tokens or 1
    w, x, state = layer_inputs(D.rank, T)
    dev = {}
    for kn, on in zip(k3cuda.KDA_WEIGHT_NAMES, W.LAYER_WEIGHTS):
        a = w[on]
        if on in W.LAYER_PROJ:
            dev[kn] = ctx.upload(a)  # bf16 bits
        else:
            dev[kn] = ctx.upload(np.ascontiguousarray(a.reshape(a.shape[0], -1) if a.ndim == 3
                                                      else a))
    del w
    dS = ctx.upload(state)
    dx = ctx.upload(x)
    dout = ctx.empty((T, E), np.float32)
    nws = ctx.kda_layer_workspace(T, E, H, Dh, K, k3cuda.BF16, k3cuda.BF16)
    ws = ctx.empty((nws,), np.uint8)

    def step():
        ctx.kda_layer(dout, dx, dev, k3cuda.BF16, T, E, H, Dh, K, -5.0, 1e-5, dS, k3cuda.BF16,
                      ws, nws)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    clk = ClockSampler(D.local)
    clk.start()
    time.sleep(0.3)
    D.barrier()
    ctx.sync()
    l0 = ctx.launches()
    t0 = clk.mark()
    ctx.record(0)
    for _ in range(args.steps):
        step()
    ctx.record(1)
    ctx.sync()
    t1 = clk.mark()
    D.barrier()
    l1 = ctx.launches()
    ms_max = D.max(ctx.elapsed_ms(0, 1))
    clocks = clk.stop(t0, t1)

    # e2e: x from page-locked host memory in, the layer output back, every step
    hx = ctx.pinned((T, E), np.float32)
    hx[...] = x
    ho = ctx.pinned((T, E), np.float32)
    L = k3cuda.lib()

    def e2e_step():
        k3cuda.check(L.k3cuda_memcpy_h2d(ctx.h, dx.ptr, hx.ctypes.data, hx.nbytes))
        step()
        k3cuda.check(L.k3cuda_memcpy_d2h(ctx.h, ho.ctypes.data, dout.ptr, ho.nbytes))

    for _ in range(3):
        e2e_step()
    ctx.sync()
    D.barrier()
    ctx.record(2)
    for _ in range(args.steps):
        e2e_step()
    ctx.record(3)
    ctx.sync()
    D.barrier()
    ms_e2e = D.max(ctx.elapsed_ms(2, 3))

    hbm, tf, src = peaks()
    per = ms_max / 1e3 / args.steps
    toks = T * args.steps * D.world
    name = f"kda_layer_T{T}"
    if T <= 8:
        alg = layer_bytes(T, E, H, Dh, K)
        roof = {"bound": "hbm", "achieved": alg / per / 1e9, "peak": hbm, "unit": "GB/s",
                "frac": alg / per / 1e9 / hbm, "peak_source": src, "traffic": None,
                "algorithmic_bytes_per_launch": alg}
    else:
        fl = layer_flops(T, E, H, Dh)
        roof = {"bound": "tensor", "achieved": fl / per / 1e12, "peak": tf, "unit": "TFLOP/s",
                "frac": fl / per / 1e12 / tf, "peak_source": src, "traffic": None,
                "algorithmic_flops_per_launch": fl}
    line = {
        "metric": f"KDA layer forward tokens/s ({name}: hidden {E}, {H} heads x {Dh}, "
                  f"bf16 weights)",
        "value": toks / (ms_max / 1e3), "unit": "tokens/s", "n_gpus": D.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded numpy weights and activations at the model's layer shape)",
        "config": {"workload": name, "tokens_per_call": T, "hidden": E, "heads": H,
                   "head_dim": Dh, "conv_k": K, "weights": "bf16",
                   "recurrence_io": "bf16", "parallelism": f"replica x{D.world}",
                   "l2": f"weights larger than L2 ({layer_weight_bytes(E, H, Dh) / 1e6:.0f} MB)"},
        "e2e": {"value": toks / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": hx.nbytes,
                "d2h_bytes_per_step": ho.nbytes},
        "roofline": roof,
        "gpu_launches": int(l1 - l0),
        "clocks": clocks,
    }
    ctx.close()
    return line


def cpu_layer_baseline(T, budget_s=10.0):
    """The reference's own k3_kda_layer (oracle/_ref) with bf16 weights on all host cores,
    on min(T, 16) tokens per call, repeated for about budget_s seconds."""
    from oracle import oracle
    if not oracle.ref_available():
        return None
    t = min(T, 16)
    wr, x, state = layer_inputs(0, t)
    E, H, Dh, K = LAYER_E, LAYER_H, LAYER_D, LAYER_K
    oracle.ref_kda_layer(x, wr, H, Dh, K, -5.0, 1e-5, state, wdt=1)
    calls, t0 = 0, time.perf_counter()
    while True:
        oracle.ref_kda_layer(x, wr, H, Dh, K, -5.0, 1e-5, state, wdt=1)
        calls += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    nth = oracle.ref().k3ref_max_threads()
    return {"value": t * calls / el, "unit": "tokens/s", "cores": nth, "kind": "reference",
            "sample": f"{calls} calls of the reference k3_kda_layer on {t} tokens each "
                      f"(bf16 weights, OpenMP matmuls and heads)"}


# ------------------------------------------------------------------- mla layer
MLA_E, MLA_H, MLA_QL = 7168, 96, 1536


def mla_layer_bytes(T, ctx_len, E=MLA_E, H=MLA_H, QL=MLA_QL):
    """bf16 weights once, the latent + rope cache of every attended position once, x/out."""
    weights = 2 * (QL * E + H * 192 * QL + 576 * E + H * 256 * 512 + E * H * 128 + H * 128 * E)
    return weights + ctx_len * 576 * 2 + 2 * T * E * 4


def mla_layer_inputs(seed, T, ctx_len, E=MLA_E, H=MLA_H, QL=MLA_QL):
    rng = np.random.default_rng(seed)
    pool = W.f32_to_bf16(rng.standard_normal(1 << 22, dtype=np.float32) * np.float32(0.02))
    mk = lambda r, c: np.resize(np.roll(pool, r), (r, c))  # noqa: E731
    w = dict(q_a=mk(QL, E), q_b=mk(H * 192, QL), kv_a=mk(576, E), kv_b=mk(H * 256, 512),
             o=mk(E, H * 128), g=mk(H * 128, E),
             q_a_norm=np.ones(QL, np.float32), kv_a_norm=np.ones(512, np.float32))
    lat = W.f32_to_bf16(rng.standard_normal((ctx_len, 512), dtype=np.float32) * np.float32(0.5))
    rope = W.f32_to_bf16(rng.standard_normal((ctx_len, 64), dtype=np.float32))
    x = rng.standard_normal((T, E), dtype=np.float32)
    return w, lat, rope, x


def bench_mla_layer(args, D: Dist):
    import k3cuda
    ctx = k3cuda.Context(D.local)
    T = args.tokens or 1
    cached = args.context if args.context is not None else 8192 - T
    cap = cached + T
    w, lat, rope, x = mla_layer_inputs(D.rank, T, cap)
    dev = {n: ctx.upload(a) for n, a in w.items()}
    dlat, drope, dx = ctx.upload(lat), ctx.upload(rope), ctx.upload(x)
    dout = ctx.empty((T, MLA_E), np.float32)
    nws = ctx.mla_layer_workspace(T, MLA_E, MLA_H, MLA_QL, cached, k3cuda.BF16)
    ws = ctx.empty((nws,), np.uint8)

    def step():  # rewrites the same T rows at cached.. every step
        ctx.mla_layer(dout, dx, dev, k3cuda.BF16, T, MLA_E, MLA_H, MLA_QL, 1e-5, dlat, drope,
                      cached, cap, ws, nws)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    clk = ClockSampler(D.local)
    clk.start()
    time.sleep(0.3)
    D.barrier()
    ctx.sync()
    l0 = ctx.launches()
    t0 = clk.mark()
    ctx.record(0)
    for _ in range(args.steps):
        step()
    ctx.record(1)
    ctx.sync()
    t1 = clk.mark()
    D.barrier()
    l1 = ctx.launches()
    ms_max = D.max(ctx.elapsed_ms(0, 1))
    clocks = clk.stop(t0, t1)
    hx = ctx.pinned((T, MLA_E), np.float32)
    hx[...] = x
    ho = ctx.pinned((T, MLA_E), np.float32)
    L = k3cuda.lib()

    def e2e_step():
        k3cuda.check(L.k3cuda_memcpy_h2d(ctx.h, dx.ptr, hx.ctypes.data, hx.nbytes))
        step()
        k3cuda.check(L.k3cuda_memcpy_d2h(ctx.h, ho.ctypes.data, dout.ptr, ho.nbytes))

    for _ in range(3):
        e2e_step()
    ctx.sync()
    D.barrier()
    ctx.record(2)
    for _ in range(args.steps):
        e2e_step()
    ctx.record(3)
    ctx.sync()
    D.barrier()
    ms_e2e = D.max(ctx.elapsed_ms(2, 3))
    hbm, tf, src = peaks()
    per = ms_max / 1e3 / args.steps
    alg = mla_layer_bytes(T, cap)
    line = {
        "metric": f"MLA layer forward tokens/s (mla_layer_T{T}_ctx{cap}: hidden {MLA_E}, "
                  f"{MLA_H} heads, bf16 weights)",
        "value": T * args.steps * D.world / (ms_max / 1e3), "unit": "tokens/s",
        "n_gpus": D.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (pooled bf16 weights, seeded latent cache and activations)",
        "config": {"workload": f"mla_layer_T{T}_ctx{cap}", "tokens_per_call": T,
                   "context": cap, "hidden": MLA_E, "heads": MLA_H, "q_lora": MLA_QL,
                   "kv_lora": 512, "qk_rope": 64, "weights": "bf16",
                   "parallelism": f"replica x{D.world}",
                   "l2": f"weights larger than L2 ({alg / 1e6:.0f} MB per call)"},
        "e2e": {"value": T * args.steps * D.world / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": hx.nbytes, "d2h_bytes_per_step": ho.nbytes},
        "roofline": {"bound": "hbm", "achieved": alg / per / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": alg / per / 1e9 / hbm, "peak_source": src, "traffic": None,
                     "algorithmic_bytes_per_launch": alg},
        "gpu_launches": int(l1 - l0), "clocks": clocks,
    }
    ctx.close()
    return line


# ----------------------------------------------------------------- moe experts
MOE_TOPK, MOE_I, MOE_L = 16, 3072, 3584


def moe_expert_bytes(k=MOE_TOPK, I=MOE_I, L=MOE_L):
    per = I * (L // 2 + L // 32)                   # one [I][L] or [L][I] MXFP4 matrix
    return 3 * k * per + k * (L + I) * 4 * 2       # + activations in and out


def moe_inputs(seed, k=MOE_TOPK, I=MOE_I, L=MOE_L):
    rng = np.random.default_rng(seed)
    pool = rng.integers(0, 256, 1 << 22, dtype=np.uint8)   # codes (values do not change time)
    w13 = [np.resize(np.roll(pool, 97 * e), (I, L // 2)) for e in range(2 * k)]
    s13 = [rng.integers(118, 128, (I, L // 32), dtype=np.uint8) for _ in range(2 * k)]
    w2 = [np.resize(np.roll(pool, 31 * e), (L, I // 2)) for e in range(k)]
    s2 = [rng.integers(118, 128, (L, I // 32), dtype=np.uint8) for _ in range(k)]
    z = rng.standard_normal((1, L)).astype(np.float32)
    act = rng.standard_normal((k, I)).astype(np.float32)
    return w13, s13, w2, s2, z, act


def bench_moe_experts(args, D: Dist):
    import k3cuda
    ctx = k3cuda.Context(D.local)
    k, I, L = MOE_TOPK, MOE_I, MOE_L
    w13, s13, w2, s2, z, act = moe_inputs(D.rank)
    d13, ds13 = [ctx.upload(a) for a in w13], [ctx.upload(a) for a in s13]
    d2, ds2 = [ctx.upload(a) for a in w2], [ctx.upload(a) for a in s2]
    dz = ctx.upload(z)
    dact = [ctx.upload(act[e:e + 1]) for e in range(k)]
    y13 = [ctx.empty((1, I), np.float32) for _ in range(2 * k)]
    y2 = [ctx.empty((1, L), np.float32) for _ in range(k)]

    def step():
        ctx.matmul_mxfp4_batch(y13, [dz] * (2 * k), d13, ds13, L, I, 1)
        ctx.matmul_mxfp4_batch(y2, dact, d2, ds2, I, L, 1)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    clk = ClockSampler(D.local)
    clk.start()
    time.sleep(0.3)
    D.barrier()
    ctx.sync()
    l0 = ctx.launches()
    t0 = clk.mark()
    ctx.record(0)
    for _ in range(args.steps):
        step()
    ctx.record(1)
    ctx.sync()
    t1 = clk.mark()
    D.barrier()
    l1 = ctx.launches()
    ms_max = D.max(ctx.elapsed_ms(0, 1))
    clocks = clk.stop(t0, t1)
    # e2e: z and the activations in from page-locked memory, every output back
    hz = ctx.pinned(z.shape, np.float32)
    hz[...] = z
    ha = ctx.pinned(act.shape, np.float32)
    ha[...] = act
    ho = ctx.pinned((3 * k, max(I, L)), np.float32)
    L_ = k3cuda.lib()

    def e2e_step():
        k3cuda.check(L_.k3cuda_memcpy_h2d(ctx.h, dz.ptr, hz.ctypes.data, hz.nbytes))
        for e in range(k):
            k3cuda.check(L_.k3cuda_memcpy_h2d(ctx.h, dact[e].ptr, ha[e:e + 1].ctypes.data, I * 4))
        step()
        for e, y in enumerate(y13 + y2):
            k3cuda.check(L_.k3cuda_memcpy_d2h(ctx.h, ho[e].ctypes.data, y.ptr, y.nbytes))

    for _ in range(3):
        e2e_step()
    ctx.sync()
    D.barrier()
    ctx.record(2)
    for _ in range(args.steps):
        e2e_step()
    ctx.record(3)
    ctx.sync()
    D.barrier()
    ms_e2e = D.max(ctx.elapsed_ms(2, 3))
    hbm, tf, src = peaks()
    per = ms_max / 1e3 / args.steps
    alg = moe_expert_bytes()
    line = {
        "metric": "MoE routed-expert decode tokens/s (16 experts x w1, w3, w2 in MXFP4)",
        "value": args.steps * D.world / (ms_max / 1e3), "unit": "tokens/s", "n_gpus": D.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic MXFP4 codes (pooled) and scales, seeded activations",
        "config": {"workload": "moe_experts_decode", "experts": k, "moe_inter": I,
                   "latent": L, "group": 32, "parallelism": f"replica x{D.world}",
                   "l2": f"weights larger than L2 ({alg / 1e6:.0f} MB per step)"},
        "e2e": {"value": args.steps * D.world / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(hz.nbytes + ha.nbytes),
                "d2h_bytes_per_step": int(sum(y.nbytes for y in y13 + y2))},
        "roofline": {"bound": "hbm", "achieved": alg / per / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": alg / per / 1e9 / hbm, "peak_source": src, "traffic": None,
                     "algorithmic_bytes_per_launch": alg},
        "gpu_launches": int(l1 - l0), "clocks": clocks,
    }
    ctx.close()
    return line


def cpu_moe_baseline(budget_s=10.0):
    """The reference's k3_matmul_mxfp4 (oracle/_ref) over the same 48 expert matrices for one
    token, OpenMP over rows on all host cores, repeated for about budget_s seconds."""
    from oracle import oracle
    if not oracle.ref_available():
        return None
    k, I, L = MOE_TOPK, MOE_I, MOE_L
    w13, s13, w2, s2, z, act = moe_inputs(0)

    def one():
        for e in range(2 * k):
            oracle.matmul_mxfp4(z, w13[e], s13[e], use_ref=True)
        for e in range(k):
            oracle.matmul_mxfp4(act[e:e + 1], w2[e], s2[e], use_ref=True)

    one()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        one()
        n += 1
    el = time.perf_counter() - t0
    return {"value": n / el, "unit": "tokens/s", "cores": oracle.ref().k3ref_max_threads(),
            "kind": "reference", "sample": f"{n} tokens x 48 expert matrices through the "
                                            f"reference k3_matmul_mxfp4"}


# ------------------------------------------------------------------ mla prefill
def mla_prefill_flops(T, H):
    """Absorbed-form FLOPs of a causal chunk from position 0: scores over 576 dims and the
    latent accumulation over 512 per (head, query, key), plus W_UK / W_UV absorption."""
    pairs = T * (T + 1) // 2
    return 2 * H * pairs * (576 + 512) + 2 * 2 * T * H * 128 * 512


def bench_mla_prefill(args, D: Dist):
    import k3cuda
    ctx = k3cuda.Context(D.local)
    T, H = args.tokens or 4096, 128
    cap = T
    c = W.mla_config4(seed=D.rank, B=1, ctx=cap, H=H)
    rng = np.random.default_rng(D.rank + 11)
    qn = W.f32_to_bf16(rng.standard_normal((T, H, 128), dtype=np.float32))
    qr = W.f32_to_bf16(rng.standard_normal((T, H, 64), dtype=np.float32))
    ct = rng.standard_normal((T, 576), dtype=np.float32)
    wn = (1.0 + 0.1 * rng.standard_normal(512)).astype(np.float32)
    d_qn, d_qr, d_ct, d_wn = ctx.upload(qn), ctx.upload(qr), ctx.upload(ct), ctx.upload(wn)
    d_lat, d_rope = ctx.upload(c["latent"]), ctx.upload(c["rope"])
    d_uk, d_uv = ctx.upload(c["w_uk"]), ctx.upload(c["w_uv"])
    seq = np.zeros(T, np.int32)
    lens = (np.arange(T) + 1).astype(np.int32)
    out = ctx.empty((T, H, 128), np.uint16)
    nws = ctx.mla_decode_workspace(lens, H)
    ws = ctx.empty((nws,), np.uint8)

    def step():
        ctx.mla_cache_append(d_lat, d_rope, d_ct, d_wn, 1e-5, 0, 0, T, 1, cap)
        ctx.mla_attend(out, d_qn, d_qr, d_lat, d_rope, d_uk, d_uv, seq, lens, 1, cap, H,
                       c["scale"], ws, nws, out_dtype=k3cuda.BF16)

    for _ in range(args.warmup):
        ctx.flush_l2()  # the first call allocates the flush buffer: keep that out of the timing
        step()
    ctx.sync()
    clk = ClockSampler(D.local)
    clk.start()
    time.sleep(0.3)
    D.barrier()
    ctx.sync()
    l0 = ctx.launches()
    t0 = clk.mark()
    ctx.record(0)
    for _ in range(args.steps):
        ctx.flush_l2()
        step()
    ctx.record(1)
    ctx.sync()
    t1 = clk.mark()
    D.barrier()
    l1 = ctx.launches()
    ms_max = D.max(ctx.elapsed_ms(0, 1))
    clocks = clk.stop(t0, t1)

    hq, hr, hc = ctx.pinned(qn.shape, np.uint16), ctx.pinned(qr.shape, np.uint16), \
        ctx.pinned(ct.shape, np.float32)
    hq[...], hr[...], hc[...] = qn, qr, ct
    ho = ctx.pinned((T, H, 128), np.uint16)
    L = k3cuda.lib()
    h2d = [(d_qn, hq), (d_qr, hr), (d_ct, hc)]

    def e2e_step():
        for dbuf, h in h2d:
            k3cuda.check(L.k3cuda_memcpy_h2d(ctx.h, dbuf.ptr, h.ctypes.data, h.nbytes))
        step()
        k3cuda.check(L.k3cuda_memcpy_d2h(ctx.h, ho.ctypes.data, out.ptr, ho.nbytes))

    for _ in range(2):
        e2e_step()
    ctx.sync()
    D.barrier()
    ctx.record(2)
    for _ in range(args.steps):
        e2e_step()
    ctx.record(3)
    ctx.sync()
    D.barrier()
    ms_e2e = D.max(ctx.elapsed_ms(2, 3))
    hbm, tf, src = peaks()
    per = ms_max / 1e3 / args.steps
    fl = mla_prefill_flops(T, H)
    line = {
        "metric": f"MLA causal prefill tokens/s (chunk of {T} tokens from position 0, 128 heads)",
        "value": T * args.steps * D.world / (ms_max / 1e3), "unit": "tokens/s",
        "n_gpus": D.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded numpy, config-4 distributions)",
        "config": {"workload": f"mla_prefill_T{T}", "tokens": T, "heads": H,
                   "cache": "latent 512 + rope 64 bf16, appended in the step",
                   "parallelism": f"replica x{D.world}",
                   "l2": "flushed before every step, flush inside the timed region (the cache "
                         "itself is L2-sized)"},
        "e2e": {"value": T * args.steps * D.world / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(sum(h.nbytes for _, h in h2d)),
                "d2h_bytes_per_step": int(ho.nbytes)},
        "roofline": {"bound": "tensor", "achieved": fl / per / 1e12, "peak": tf,
                     "unit": "TFLOP/s", "frac": fl / per / 1e12 / tf, "peak_source": src,
                     "traffic": None, "algorithmic_flops_per_launch": fl,
                     "flops_form": "absorbed (latent) form"},
        "gpu_launches": int(l1 - l0),  # the L2 flush is a memset, not a kernel
        "clocks": clocks,
    }
    ctx.close()
    return line


# -------------------------------------------------------------- reference arm
def ref_decode_step_sampler(args):
    """The reference's k3_kda_step over config 1, each step a sample of the batch sized so
    the whole run stays within a couple of minutes."""
    from oracle import oracle
    B, H, d = DECODE_B, DECODE_H, DECODE_D
    c = W.kda_config1(B=B, H=H, d=d)
    nth = oracle.ref().k3ref_max_threads()
    S = c["state"].copy()
    t0 = time.perf_counter()
    oracle.kda_decode(S, c["q"], c["k"], c["v"], c["g"], c["beta"], use_ref=True, nthreads=nth)
    full = time.perf_counter() - t0
    total = args.steps + args.warmup
    frac = min(1.0, 120.0 / max(full * total, 1e-9))
    nb = max(1, int(B * frac))
    sub = {x: np.ascontiguousarray(c[x][:nb]) for x in ("q", "k", "v", "g", "beta")}
    Ss = np.ascontiguousarray(S[:nb])
    for _ in range(args.warmup):
        _, Ss = oracle.kda_decode(Ss, sub["q"], sub["k"], sub["v"], sub["g"], sub["beta"],
                                  use_ref=True, nthreads=nth)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _, Ss = oracle.kda_decode(Ss, sub["q"], sub["k"], sub["v"], sub["g"], sub["beta"],
                                  use_ref=True, nthreads=nth)
    el = time.perf_counter() - t0
    return nb * args.steps / el, el, nth, (f"{nb} of {B} sequences x {H} heads per step "
                                            f"through the reference k3_kda_step (OpenMP over "
                                            f"streams)")


def bench_reference(args, D: Dist):
    """The reference's own C on the host cores (oracle/_ref/libk3ref.so, its unmodified
    k3_ops.c; for config 4 the C restatement of its attention loop), for the same workload,
    metric and unit as our arm. Rank 0 only."""
    from oracle import oracle
    if not oracle.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libk3ref.so was not built"}
    wl = args.workload
    base = {"impl": "reference", "n_gpus": D.world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "vs_baseline": None, "dtype": "mixed",
            "data": "synthetic", "unit": "tokens/s"}
    if wl == "decode":
        value, el, nth, sample = ref_decode_step_sampler(args)
        line = dict(base, metric="KDA recurrent decode tokens/s (BASELINE config 1: B=256, "
                                 "H=32, d=128)",
                    value=value, ms_per_step=el * 1e3 / args.steps, scaling="weak",
                    config=decode_config(DECODE_B, DECODE_H, DECODE_D))
        cpu = {"value": value, "unit": "tokens/s", "cores": nth, "kind": "reference",
               "sample": sample}
        if not args.no_subrecords:
            for key, which in (("prefill_cfg2", "cfg2"), ("varlen_cfg3", "cfg3")):
                H = PREFILL[which]["H"]
                cb = cpu_prefill_baseline(prefill_sample(which), H)
                line[key] = {"metric": f"KDA chunked prefill tokens/s "
                                       f"({PREFILL[which]['name']})",
                             "value": cb["value"], "unit": "tokens/s", "cpu_baseline": cb}
            cb = cpu_mla_baseline(W.mla_config4(B=2))
            line["mla_cfg4"] = {"metric": "MLA absorbed decode tokens/s (BASELINE config 4)",
                                "value": cb["value"], "unit": "tokens/s", "cpu_baseline": cb}
    elif wl in ("prefill", "varlen"):
        which = "cfg2" if wl == "prefill" else "cfg3"
        H = PREFILL[which]["H"]
        budget = 2.0 * max(1, args.steps) / 10
        cpu = cpu_prefill_baseline(prefill_sample(which), H, budget_s=budget)
        value = cpu["value"]
        T = args.tokens or (32768 if which == "cfg2" else int(W.config3_cu_seqlens()[-1]))
        line = dict(base, metric=f"KDA chunked prefill tokens/s ({PREFILL[which]['name']})",
                    value=value, ms_per_step=T / value * 1e3, scaling="strong",
                    config={"workload": PREFILL[which]["name"], "tokens": T, "heads_total": H,
                            "d": 128, "chunk": 64})
    elif wl == "mla":
        c = W.mla_config4(B=2)
        cpu = cpu_mla_baseline(c, budget_s=2.0 * max(1, args.steps) / 10)
        value = cpu["value"]
        line = dict(base, metric="MLA absorbed decode tokens/s (BASELINE config 4)",
                    value=value, ms_per_step=64 / value * 1e3, scaling="strong",
                    config={"workload": "mla_decode_config4", "batch": 64, "ctx": 8192,
                            "heads": 128})
    else:
        return {"impl": "reference",
                "unavailable": f"the reference arm covers decode, prefill, varlen and mla; "
                               f"{wl} is timed beside our arm as its cpu_baseline"}
    line["cpu_baseline"] = cpu
    line["e2e"] = {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "varlen", "mla", "mla_prefill", "layer",
                             "moe_experts", "mla_layer"])
    ap.add_argument("--context", type=int, default=None,
                    help="mla_layer: positions already in the cache before the new tokens")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="decode: print the headline alone, without the config-2/3/4 records")
    ap.add_argument("--io", default="bf16", choices=["bf16", "f32"],
                    help="prefill / varlen: the q/k/v/o element type (f32: the path the fp32 "
                         "drop-ins use; one GPU)")
    ap.add_argument("--batch", type=int, default=None,
                    help="mla: sequences per GPU in place of 64 / N (a profiling case: the "
                         "per-GPU share of config 4 at more GPUs)")
    ap.add_argument("--tokens", type=int, default=None,
                    help="prefill: sequence length in place of config 2's 32768 (a small case "
                         "for kernel profiling; not a headline number); layer: tokens per call")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    D = Dist()
    if args.impl == "reference":
        if D.rank == 0:
            print(json.dumps(bench_reference(args, D)), flush=True)
        D.close()
        return
    if args.workload == "decode":
        line = bench_decode(args, D)
        if not args.no_subrecords:
            # the other BASELINE configurations, each a record of its own in the same line
            line["prefill_cfg2"] = guarded(prefill_record, args, D, "cfg2")
            line["varlen_cfg3"] = guarded(prefill_record, args, D, "cfg3")
            line["mla_cfg4"] = guarded(mla_record, args, D)
    elif args.workload in ("prefill", "varlen"):
        which = "cfg2" if args.workload == "prefill" else "cfg3"
        line = prefill_record(args, D, which, tokens=args.tokens)
        line["vs_baseline"] = None
        line["data"] = "synthetic (seeded numpy: BASELINE config distributions)"
    elif args.workload == "layer":
        line = bench_layer(args, D)
    elif args.workload == "mla_prefill":
        line = bench_mla_prefill(args, D)
    elif args.workload == "moe_experts":
        line = bench_moe_experts(args, D)
    elif args.workload == "mla_layer":
        line = bench_mla_layer(args, D)
    else:
        line = mla_record(args, D)
        line["vs_baseline"] = None
        line["data"] = "synthetic (seeded numpy: BASELINE config-4 distributions)"
    if D.rank == 0:
        if args.workload == "decode" and D.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_decode_baseline(DECODE_B, DECODE_H, DECODE_D)
        if args.workload == "layer" and D.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_layer_baseline(args.tokens or 1)
        if args.workload == "moe_experts" and D.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_moe_baseline()
        print(json.dumps(line), flush=True)
    D.close()


if __name__ == "__main__":
    main()
