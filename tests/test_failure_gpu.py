"""Failure detection in the forms this pool allows: no test faults, traps or hangs a GPU.

* A device-side bounded wait runs out on purpose (a barrier nothing completes, under a
  bound of a few thousand microseconds): the kernel records its code and returns, the next
  k3cuda_sync reports K3CUDA_ERR_TIMEOUT, and the context keeps computing correct results.
* A rank leaves between steps (no kernel or collective of its own in flight): the other
  rank's next collective call ends under the communicator's deadline with
  ncclCommAbort and an error status instead of a hang, and its context keeps working on
  single-GPU calls. Two processes on two GPUs, NVLS off; skipped on a one-GPU box.
"""
import json
import os
import socket
import time

import numpy as np
import pytest

import workloads as W

pytestmark = pytest.mark.gpu


def _small_decode(c, seed):
    """One KDA decode step through the context, checked against the oracle."""
    from oracle import oracle
    rng = np.random.default_rng(seed)
    B, H, d = 3, 2, 128
    t = W.kda_tokens(rng, B, H, d, d, bf16=True)
    S = rng.standard_normal((B, H, d, d), dtype=np.float32) * np.float32(0.02)
    bf = W.f32_to_bf16
    dS = c.upload(S)
    dq, dk, dv = c.upload(bf(t["q"])), c.upload(bf(t["k"])), c.upload(bf(t["v"]))
    dg, db = c.upload(t["g"]), c.upload(t["beta"])
    do = c.empty((B, H, d), np.uint16)
    c.kda_decode(dS, do, dq, dk, dv, dg, db, B, H, d, d, 1.0 / np.sqrt(np.float32(d)))
    c.sync()
    o_ref, S_ref = oracle.kda_decode(S, t["q"], t["k"], t["v"], t["g"], t["beta"])
    return (W.rel_fro(W.bf16_to_f32(do.numpy()), o_ref), W.rel_fro(dS.numpy(), S_ref))


def test_device_wait_runs_out_and_the_context_stays_usable():
    import k3cuda
    c = k3cuda.Context(0)
    try:
        c.set_wait_limit(2_000_000)  # about a millisecond at the B200's clocks
        t0 = time.perf_counter()
        c.wait_selftest()
        with pytest.raises(k3cuda.K3CudaError) as ei:
            c.sync()
        assert ei.value.code == k3cuda.ERR_TIMEOUT
        assert "0x5e1f" in str(ei.value).lower()
        assert time.perf_counter() - t0 < 10.0
        c.sync()  # the error word was cleared by the report
        c.set_wait_limit(0)  # back to the default bound
        e_o, e_S = _small_decode(c, 5)
        assert e_o < 5e-3 and e_S < 2e-3
    finally:
        c.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _leaver_main(rank, port, outdir):
    """Rank 1 runs one gathered step and leaves; rank 0 then calls the next step alone."""
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [root, os.path.join(root, "kimi-k3-in-c_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import k3cuda
    import sharding
    import workloads as W_
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60))
    obj = [k3cuda.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    c = k3cuda.Context(rank)
    c.comm_set_timeout(4000)
    c.comm_init(2, rank, obj[0])
    H = 4
    rng = np.random.default_rng(3)
    cu = np.array([0, 90, 200], np.int32)
    t = W_.kda_tokens(rng, int(cu[-1]), H, 128, 128, bf16=True)
    hs = sharding.head_shard(H, 2, rank)
    Hl = hs.stop - hs.start
    full = c.empty((int(cu[-1]), H, 128), np.uint16)
    c.comm_register_full(full)
    S = c.empty((2, Hl, 128, 128), np.float32)
    nws = c.kda_prefill_workspace(cu, Hl, 128, 128)
    ws = c.empty((nws,), np.uint8)
    args = [c.upload(np.ascontiguousarray(W_.f32_to_bf16(t[x][:, hs]))) for x in ("q", "k", "v")]
    args += [c.upload(np.ascontiguousarray(t["g"][:, hs])),
             c.upload(np.ascontiguousarray(t["beta"][:, hs]))]
    qs = 1.0 / np.sqrt(128.0)
    S.zero()
    c.kda_prefill_gathered(S, *args, cu, Hl, 128, 128, qs, ws, nws)
    c.sync()  # step 1 complete on this rank: nothing of it is in flight any more
    dist.barrier()
    if rank == 1:
        # leave between steps, without tearing anything down (as a crashed process would)
        open(os.path.join(outdir, "left"), "w").close()
        os._exit(0)
    while not os.path.exists(os.path.join(outdir, "left")):
        time.sleep(0.05)
    time.sleep(1.0)
    res = {}
    t0 = time.perf_counter()
    try:
        S.zero()
        c.kda_prefill_gathered(S, *args, cu, Hl, 128, 128, qs, ws, nws)
        c.sync()
        res["first"] = "no error"
    except k3cuda.K3CudaError as e:
        res["first"] = e.code
    res["seconds"] = time.perf_counter() - t0
    try:
        c.kda_prefill_gathered(S, *args, cu, Hl, 128, 128, qs, ws, nws)
        res["second"] = "no error"
    except k3cuda.K3CudaError as e:
        res["second"] = e.code
    # the context still runs single-GPU work: an unsharded prefill of this rank's heads
    o = c.empty((int(cu[-1]), Hl, 128), np.uint16)
    S.zero()
    c.kda_prefill(S, o, *args, cu, Hl, 128, 128, qs, ws, nws)
    c.sync()
    res["after"] = bool(np.isfinite(W_.bf16_to_f32(o.numpy())).all())
    c.close()
    with open(os.path.join(outdir, "rank0.json"), "w") as f:
        json.dump(res, f)
    os._exit(0)  # the gloo group lost its peer: skip its teardown


def test_peer_leaves_between_steps_and_the_collective_aborts(tmp_path):
    import multiprocessing as mp

    import k3cuda
    if k3cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_leaver_main, args=(r, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    with open(tmp_path / "rank0.json") as f:
        res = json.load(f)
    assert res["first"] in (k3cuda.ERR_TIMEOUT, k3cuda.ERR_NCCL), res
    assert res["seconds"] < 60, res
    assert res["second"] == k3cuda.ERR_STATE, res
    assert res["after"] is True, res
