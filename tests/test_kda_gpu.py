"""KDA decode and chunked prefill on the B200 against the oracle and the golden vectors.

Tolerances (relative Frobenius error, written per test): 2e-3 for fp32 inputs and for the
fp32 state, 5e-3 where inputs or outputs are bf16 -- the bar of the hot-path contract.
Inputs are seeded; bf16 tensors are rounded on the host, and the oracle consumes the exact
widened values, so both sides see identical numbers.
"""
import numpy as np
import pytest

import k3cuda
import workloads as W
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL_F32 = 2e-3
TOL_BF16 = 5e-3


def _bf(x):
    return W.f32_to_bf16(x)


def run_decode(ctx, S, q, k, v, gate, beta, io=k3cuda.BF16, gate_mode=k3cuda.GATE_LOG,
               q_scale=None):
    B, H, dk = q.shape
    dv = v.shape[2]
    if q_scale is None:
        q_scale = 1.0 / np.sqrt(np.float32(dk))
    conv = _bf if io == k3cuda.BF16 else (lambda x: np.ascontiguousarray(x, np.float32))
    dS = ctx.upload(np.ascontiguousarray(S, np.float32))
    dq, dk_, dv_ = ctx.upload(conv(q)), ctx.upload(conv(k)), ctx.upload(conv(v))
    dg, db = ctx.upload(np.ascontiguousarray(gate, np.float32)), ctx.upload(
        np.ascontiguousarray(beta, np.float32))
    do = ctx.empty((B, H, dv), np.uint16 if io == k3cuda.BF16 else np.float32)
    ctx.kda_decode(dS, do, dq, dk_, dv_, dg, db, B, H, dk, dv, q_scale, io, gate_mode)
    o = do.numpy()
    if io == k3cuda.BF16:
        o = W.bf16_to_f32(o)
    return o, dS.numpy()


def run_prefill(ctx, q, k, v, g, beta, cu, S0=None, io=k3cuda.BF16, gate_mode=k3cuda.GATE_LOG,
                with_state=True):
    T, H, dk = q.shape
    dv = v.shape[2]
    nseq = len(cu) - 1
    conv = _bf if io == k3cuda.BF16 else (lambda x: np.ascontiguousarray(x, np.float32))
    dq, dk_, dv_ = ctx.upload(conv(q)), ctx.upload(conv(k)), ctx.upload(conv(v))
    dg, db = ctx.upload(np.ascontiguousarray(g, np.float32)), ctx.upload(
        np.ascontiguousarray(beta, np.float32))
    dS = None
    if with_state:
        S0 = np.zeros((nseq, H, dk, dv), np.float32) if S0 is None else S0
        dS = ctx.upload(np.ascontiguousarray(S0, np.float32))
    do = ctx.empty((T, H, dv), np.uint16 if io == k3cuda.BF16 else np.float32)
    nws = ctx.kda_prefill_workspace(cu, H, dk, dv)
    ws = ctx.empty((max(nws, 1),), np.uint8)
    ctx.kda_prefill(dS, do, dq, dk_, dv_, dg, db, cu, H, dk, dv, 1.0 / np.sqrt(np.float32(dk)),
                    ws, nws, io, gate_mode)
    o = do.numpy()
    if io == k3cuda.BF16:
        o = W.bf16_to_f32(o)
    return o, (dS.numpy() if dS is not None else None)


# --------------------------------------------------------------------------- decode
@pytest.mark.parametrize("name", ["kda_recur1", "kda_recur8"])
def test_decode_matches_reference_fixture(ctx, golden, name):
    """The reference's own fixture (H=4, d=16, alpha given, q_scale 0.25), token by token
    through the general decode kernel, fp32 I/O."""
    d = golden(name)
    T, H, dk = d["q"].shape
    S = np.zeros((1, H, dk, dk), np.float32)
    outs = []
    for t in range(T):
        o, S2 = run_decode(ctx, S, d["q"][t:t + 1], d["k"][t:t + 1], d["v"][t:t + 1],
                           d["alpha"][t:t + 1], d["beta"][t:t + 1], io=k3cuda.F32,
                           gate_mode=k3cuda.GATE_ALPHA, q_scale=float(d["q_scale"]))
        S = S2
        outs.append(o[0])
    assert W.rel_fro(np.stack(outs), d["out"]) < 1e-5
    assert W.rel_fro(S[0], d["state_out"]) < 1e-5


@pytest.mark.parametrize("dk", [64, 128])
@pytest.mark.parametrize("io", [k3cuda.F32, k3cuda.BF16])
def test_decode_fast_path_vs_reference_c(ctx, dk, io):
    rng = np.random.default_rng(11 + dk)
    B, H, dv = 6, 5, 128
    t = W.kda_tokens(rng, B, H, dk, dv, bf16=(io == k3cuda.BF16))
    S = rng.standard_normal((B, H, dk, dv), dtype=np.float32) * np.float32(0.02)
    o, S2 = run_decode(ctx, S, t["q"], t["k"], t["v"], t["g"], t["beta"], io=io)
    use_ref = oracle.ref_available()
    o_ref, S_ref = oracle.kda_decode(S, t["q"], t["k"], t["v"], t["g"], t["beta"], use_ref=use_ref)
    tol = TOL_BF16 if io == k3cuda.BF16 else TOL_F32
    assert W.rel_fro(o, o_ref) < tol
    assert W.rel_fro(S2, S_ref) < 1e-5  # the state stays fp32 end to end


def test_decode_config1_full_size(ctx):
    """BASELINE config 1 at full size: B=256, H=32, d=128, bf16 q/k/v/o, fp32 state."""
    c = W.kda_config1()
    o, S2 = run_decode(ctx, c["state"], c["q"], c["k"], c["v"], c["g"], c["beta"])
    o_ref, S_ref = oracle.kda_decode(c["state"], c["q"], c["k"], c["v"], c["g"], c["beta"],
                                     nthreads=oracle.max_threads())
    assert W.rel_fro(o, o_ref) < TOL_BF16
    assert W.rel_fro(S2, S_ref) < TOL_F32
    # a size-independent property: a second step equals two oracle steps
    o2, S3 = run_decode(ctx, S2, c["q"], c["k"], c["v"], c["g"], c["beta"])
    o2_ref, S3_ref = oracle.kda_decode(S_ref, c["q"], c["k"], c["v"], c["g"], c["beta"],
                                       nthreads=oracle.max_threads())
    assert W.rel_fro(S3, S3_ref) < TOL_F32 and W.rel_fro(o2, o2_ref) < TOL_BF16


def test_decode_alpha_mode_equals_log_mode(ctx):
    rng = np.random.default_rng(3)
    t = W.kda_tokens(rng, 4, 3, 128, 128, bf16=False)
    S = rng.standard_normal((4, 3, 128, 128), dtype=np.float32) * np.float32(0.02)
    o1, S1 = run_decode(ctx, S, t["q"], t["k"], t["v"], t["g"], t["beta"], io=k3cuda.F32)
    o2, S2 = run_decode(ctx, S, t["q"], t["k"], t["v"], np.exp(t["g"]), t["beta"], io=k3cuda.F32,
                        gate_mode=k3cuda.GATE_ALPHA)
    assert W.rel_fro(o1, o2) < 1e-6 and W.rel_fro(S1, S2) < 1e-6


def _host_step(ctx, dS, t, io, gate_mode, slices, pinned, n_streams, H, dk, dv, st=None):
    """One k3cuda_kda_decode_host call from host arrays (staging `st`, or a new buffer);
    returns the host output array and the staging buffer. Valid after ctx.sync()."""
    conv = _bf if io == k3cuda.BF16 else (lambda x: np.ascontiguousarray(x, np.float32))
    ety = np.uint16 if io == k3cuda.BF16 else np.float32
    src = {"q": conv(t["q"]), "k": conv(t["k"]), "v": conv(t["v"]),
           "g": np.ascontiguousarray(t["g"], np.float32),
           "beta": np.ascontiguousarray(t["beta"], np.float32)}
    if pinned:
        for name in list(src):
            a = ctx.pinned(src[name].shape, src[name].dtype)
            a[...] = src[name]
            src[name] = a
        ho = ctx.pinned((n_streams, H, dv), ety)
    else:
        ho = np.empty((n_streams, H, dv), ety)
    n = ctx.kda_decode_host_workspace(n_streams, H, dk, dv, io)
    st = ctx.empty((n,), np.uint8) if st is None else st
    ctx.kda_decode_host(dS, ho, src["q"], src["k"], src["v"], src["g"], src["beta"], n_streams,
                        H, dk, dv, 1.0 / np.sqrt(np.float32(dk)), st, n, io, gate_mode,
                        slices=slices)
    return ho, st


@pytest.mark.parametrize("slices", [-1, 0, 1, 3, 7, 16])
def test_decode_host_buffers_equal_device_path(ctx, slices):
    """k3cuda_kda_decode_host (host tensors in and out) gives the device-buffer step bit for
    bit: in place over PCIe (-1, and 0 with page-locked buffers), and through copies
    pipelined over batch slices on every split (uneven, more slices than sequences)."""
    rng = np.random.default_rng(41 + slices)
    B, H, d = 37, 4, 128
    t = W.kda_tokens(rng, B, H, d, d, bf16=True)
    S = rng.standard_normal((B, H, d, d), dtype=np.float32) * np.float32(0.02)
    o_dev, S_dev = run_decode(ctx, S, t["q"], t["k"], t["v"], t["g"], t["beta"])
    dS = ctx.upload(S)
    ho, _ = _host_step(ctx, dS, t, k3cuda.BF16, k3cuda.GATE_LOG, slices, True, B, H, d, d)
    ctx.sync()
    assert np.array_equal(W.bf16_to_f32(np.array(ho)), o_dev)
    assert np.array_equal(dS.numpy(), S_dev)


def test_decode_host_in_place_refuses_pageable_memory(ctx):
    """In-place mode needs page-locked buffers: pageable ones are an argument error, with
    nothing launched."""
    rng = np.random.default_rng(8)
    B, H, d = 2, 2, 128
    t = W.kda_tokens(rng, B, H, d, d, bf16=True)
    dS = ctx.upload(np.zeros((B, H, d, d), np.float32))
    n0 = ctx.launches()
    with pytest.raises(k3cuda.K3CudaError):
        _host_step(ctx, dS, t, k3cuda.BF16, k3cuda.GATE_LOG, -1, False, B, H, d, d)
    assert ctx.launches() == n0


def test_decode_host_pageable_fp32_alpha_consecutive_steps(ctx):
    """Pageable host arrays, fp32 I/O, alpha gate, dk=64, two host steps enqueued back to
    back (the second's copies must wait for the first's kernels): equal to two device steps
    bit for bit, and to the oracle within the fp32 bar."""
    rng = np.random.default_rng(5)
    B, H, dk, dv = 9, 3, 64, 128
    S = rng.standard_normal((B, H, dk, dv), dtype=np.float32) * np.float32(0.02)
    ts = [W.kda_tokens(rng, B, H, dk, dv, bf16=False) for _ in range(2)]
    logg = [t["g"] for t in ts]
    for t in ts:
        t["g"] = np.exp(t["g"])
    S_dev, o_dev = S, []
    for t in ts:
        o, S_dev = run_decode(ctx, S_dev, t["q"], t["k"], t["v"], t["g"], t["beta"],
                              io=k3cuda.F32, gate_mode=k3cuda.GATE_ALPHA)
        o_dev.append(o)
    dS = ctx.upload(S)
    ho1, st = _host_step(ctx, dS, ts[0], k3cuda.F32, k3cuda.GATE_ALPHA, 2, False, B, H, dk, dv)
    ho2, _ = _host_step(ctx, dS, ts[1], k3cuda.F32, k3cuda.GATE_ALPHA, 3, False, B, H, dk, dv,
                        st=st)  # the same staging buffer: ordered behind the first step
    ctx.sync()
    assert np.array_equal(ho1, o_dev[0]) and np.array_equal(ho2, o_dev[1])
    assert np.array_equal(dS.numpy(), S_dev)
    S_ref = S
    for t, g, ho in zip(ts, logg, (ho1, ho2)):
        o_ref, S_ref = oracle.kda_decode(S_ref, t["q"], t["k"], t["v"], g, t["beta"])
        assert W.rel_fro(ho, o_ref) < TOL_F32


# -------------------------------------------------------------------------- prefill
def test_config0_prefill_then_decode_matches_reference_c(ctx, golden):
    """chunked prefill of 256 tokens, then 32 decode steps, against the
    reference C recurrence over all 288 tokens (fp32, H=4, d=64)."""
    d = golden("cfg0_kda")
    Tp = 256
    o_p, S = run_prefill(ctx, d["q"][:Tp], d["k"][:Tp], d["v"][:Tp], d["g"][:Tp],
                         d["beta"][:Tp], np.array([0, Tp], np.int32), io=k3cuda.F32)
    outs = [o_p]
    for t in range(Tp, Tp + 32):
        o, S = run_decode(ctx, S, d["q"][t][None], d["k"][t][None], d["v"][t][None],
                          d["g"][t][None], d["beta"][t][None], io=k3cuda.F32)
        outs.append(o)
    out = np.concatenate(outs, axis=0)
    assert W.rel_fro(out, d["out"]) < TOL_F32
    assert W.rel_fro(S, d["state_out"]) < TOL_F32
    assert W.rel_fro(out[:Tp], d["out"][:Tp]) < TOL_F32


RAGGED = [0, 1, 63, 64, 65, 0, 130, 7, 200]


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_varlen_ragged_bf16(ctx, d):
    """Packed sequences with empty, single-token, exact-chunk and partial-chunk lengths,
    a nonzero initial state, bf16 q/k/v/o."""
    rng = np.random.default_rng(7 + d)
    H = 3
    cu = np.concatenate([[0], np.cumsum(RAGGED)]).astype(np.int32)
    t = W.kda_tokens(rng, int(cu[-1]), H, d, d, bf16=True)
    S0 = rng.standard_normal((len(RAGGED), H, d, d), dtype=np.float32) * np.float32(0.05)
    o, S = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu, S0=S0)
    o_ref, S_ref = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu, state=S0,
                                         nthreads=oracle.max_threads())
    # bf16 inputs: the 5e-3 bar applies to the outputs and to the final state
    assert W.rel_fro(o, o_ref) < TOL_BF16
    assert W.rel_fro(S, S_ref) < TOL_BF16
    for n in range(len(RAGGED)):  # every sequence on its own, not only in aggregate
        a, b = cu[n], cu[n + 1]
        if b > a:
            assert W.rel_fro(o[a:b], o_ref[a:b]) < TOL_BF16, n
        assert W.rel_fro(S[n], S_ref[n]) < TOL_BF16, n
    assert np.array_equal(S[0], S0[0]) and np.array_equal(S[5], S0[5])  # empty: untouched


def test_prefill_many_streams_bf16(ctx):
    """Many (sequence, head) streams (the config-3 shape class: more scan CTAs than SMs),
    ragged lengths, nonzero initial state."""
    rng = np.random.default_rng(17)
    H, d = 16, 128
    lens = [1, 64, 100, 130, 7, 0, 257, 64, 65, 33]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    t = W.kda_tokens(rng, int(cu[-1]), H, d, d, bf16=True)
    S0 = rng.standard_normal((len(lens), H, d, d), dtype=np.float32) * np.float32(0.05)
    o, S = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu, S0=S0)
    o_ref, S_ref = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu, state=S0,
                                         nthreads=oracle.max_threads())
    assert W.rel_fro(o, o_ref) < TOL_BF16
    assert W.rel_fro(S, S_ref) < TOL_BF16
    for n in range(len(lens)):
        a, b = cu[n], cu[n + 1]
        if b > a:
            assert W.rel_fro(o[a:b], o_ref[a:b]) < TOL_BF16, n
        assert W.rel_fro(S[n], S_ref[n]) < TOL_BF16, n


def test_prefill_without_state_and_alpha_gate(ctx):
    rng = np.random.default_rng(21)
    H, d = 2, 128
    cu = np.array([0, 150, 300], np.int32)
    t = W.kda_tokens(rng, 300, H, d, d, bf16=False)
    o1, _ = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu, io=k3cuda.F32,
                        with_state=False)
    o2, _ = run_prefill(ctx, t["q"], t["k"], t["v"], np.exp(t["g"]), t["beta"], cu,
                        io=k3cuda.F32, gate_mode=k3cuda.GATE_ALPHA, with_state=False)
    o_ref, _ = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu,
                                     nthreads=oracle.max_threads())
    assert W.rel_fro(o1, o_ref) < TOL_F32 and W.rel_fro(o2, o_ref) < TOL_F32


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_extreme_decay_takes_the_exact_path(ctx, d):
    """Channels decaying by e^-30 per token overflow a 15-token anchor; the kernel must form
    those sub-block entries directly and still match (fp32; d = 128 runs the tensor-core
    scan on the intra-chunk kernel's hi/lo operands)."""
    rng = np.random.default_rng(9)
    H, T = 2, 128
    t = W.kda_tokens(rng, T, H, d, d, bf16=False)
    t["g"][:, :, :8] = -30.0
    t["g"][:, :, 8:16] = 0.0  # alpha == 1 exactly: perfect retention is legitimate
    cu = np.array([0, T], np.int32)
    o, S = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu, io=k3cuda.F32)
    o_ref, S_ref = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu)
    assert np.all(np.isfinite(o)) and np.all(np.isfinite(S))
    assert W.rel_fro(o, o_ref) < TOL_F32 and W.rel_fro(S, S_ref) < TOL_F32


# fp32 q/k/v/o at d = 128 run the tensor-core scan with every operand split into bf16 hi + lo
# (three MMAs per product): about 2^-16 relative error per product, so this bar sits far
# below what single bf16 operands reach (~4e-3) and far above fp32 rounding.
TOL_SPLIT = 1e-4


def test_prefill_varlen_ragged_fp32_tensor_core(ctx):
    """fp32 I/O, d = 128: empty, single-token, exact-chunk and partial-chunk sequences with a
    nonzero initial state, every sequence checked on its own at the split-precision bar."""
    rng = np.random.default_rng(41)
    H, d = 3, 128
    cu = np.concatenate([[0], np.cumsum(RAGGED)]).astype(np.int32)
    t = W.kda_tokens(rng, int(cu[-1]), H, d, d, bf16=False)
    S0 = rng.standard_normal((len(RAGGED), H, d, d), dtype=np.float32) * np.float32(0.05)
    o, S = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu, S0=S0,
                       io=k3cuda.F32)
    o_ref, S_ref = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu, state=S0,
                                         nthreads=oracle.max_threads())
    assert W.rel_fro(o, o_ref) < TOL_SPLIT
    assert W.rel_fro(S, S_ref) < TOL_SPLIT
    for n in range(len(RAGGED)):
        a, b = cu[n], cu[n + 1]
        if b > a:
            assert W.rel_fro(o[a:b], o_ref[a:b]) < TOL_SPLIT, n
        assert W.rel_fro(S[n], S_ref[n]) < TOL_SPLIT, n
    assert np.array_equal(S[0], S0[0]) and np.array_equal(S[5], S0[5])  # empty: untouched


def test_prefill_fp32_unaligned_pointers_match_aligned(ctx):
    """fp32 v, o and state 4 bytes off a 16-byte boundary (the tensor-core scan then takes
    its scalar-access form): the results equal the aligned call's bit for bit."""
    rng = np.random.default_rng(43)
    H, d = 2, 128
    cu = np.array([0, 100, 100, 230], np.int32)
    T = int(cu[-1])
    t = W.kda_tokens(rng, T, H, d, d, bf16=False)
    S0 = rng.standard_normal((3, H, d, d), dtype=np.float32) * np.float32(0.05)
    o_al, S_al = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu, S0=S0,
                             io=k3cuda.F32)
    L = k3cuda.lib()

    def shifted(a):  # a device copy of `a` starting 4 bytes past a 16-byte boundary
        a = np.ascontiguousarray(a, np.float32)
        buf = ctx.empty((a.size + 4,), np.float32)
        k3cuda.check(L.k3cuda_memcpy_h2d(ctx.h, buf.ptr + 4, a.ctypes.data, a.nbytes))
        return buf, buf.ptr + 4

    def fetch(p, shape):
        out = np.empty(shape, np.float32)
        k3cuda.check(L.k3cuda_memcpy_d2h(ctx.h, out.ctypes.data, p, out.nbytes))
        return out

    dq, dk_, dg, db = (ctx.upload(np.ascontiguousarray(t[x], np.float32))
                       for x in ("q", "k", "g", "beta"))
    vb, vp = shifted(t["v"])
    sb, sp = shifted(S0)
    ob, op = shifted(np.zeros((T, H, d), np.float32))
    nws = ctx.kda_prefill_workspace(cu, H, d, d)
    ws = ctx.empty((nws,), np.uint8)
    ctx.kda_prefill(sp, op, dq, dk_, vp, dg, db, cu, H, d, d, 1.0 / np.sqrt(np.float32(d)), ws,
                    nws, k3cuda.F32)
    ctx.sync()
    assert np.array_equal(fetch(op, (T, H, d)), o_al)
    assert np.array_equal(fetch(sp, S0.shape), S_al)


def test_prefill_extreme_decay_bf16_tensor_core(ctx):
    """The same overflow case through the tensor-core path (bf16, d=128): the flagged
    sub-blocks' columns of Akk/Aqk are recomputed exactly inside the intra-chunk kernel."""
    rng = np.random.default_rng(10)
    H, d, T = 2, 128, 200
    t = W.kda_tokens(rng, T, H, d, d, bf16=True)
    t["g"][:, :, :8] = -30.0
    t["g"][:, :, 8:16] = 0.0
    cu = np.array([0, 70, T], np.int32)
    S0 = rng.standard_normal((2, H, d, d), dtype=np.float32) * np.float32(0.05)
    o, S = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu, S0=S0)
    o_ref, S_ref = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu, state=S0,
                                         nthreads=oracle.max_threads())
    assert np.all(np.isfinite(o)) and np.all(np.isfinite(S))
    assert W.rel_fro(o, o_ref) < TOL_BF16 and W.rel_fro(S, S_ref) < TOL_BF16


def test_prefill_alpha_gate_bf16_tensor_core(ctx):
    """Gates given as decay factors alpha (not log-decay) through the tensor-core path."""
    rng = np.random.default_rng(23)
    H, d = 4, 128
    cu = np.array([0, 37, 200, 330], np.int32)
    t = W.kda_tokens(rng, 330, H, d, d, bf16=True)
    o, S = run_prefill(ctx, t["q"], t["k"], t["v"], np.exp(t["g"]), t["beta"], cu,
                       gate_mode=k3cuda.GATE_ALPHA)
    o_ref, S_ref = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu,
                                         state=np.zeros((3, H, d, d), np.float32),
                                         nthreads=oracle.max_threads())
    assert W.rel_fro(o, o_ref) < TOL_BF16 and W.rel_fro(S, S_ref) < TOL_BF16


def test_prefill_config2_length_fp32_tensor_core(ctx):
    """fp32 I/O over config 2's sequence length (512 chunks in one tensor-core scan, the state
    carried as bf16 hi/lo between chunks): the split-precision error does not grow along the
    chain."""
    rng = np.random.default_rng(2)
    T, H, d = 32768, 2, 128
    t = W.kda_tokens(rng, T, H, d, d, bf16=False)
    cu = np.array([0, T], np.int32)
    o, S = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu, io=k3cuda.F32)
    o_ref, S_ref = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu,
                                         nthreads=oracle.max_threads())
    assert W.rel_fro(o, o_ref) < TOL_SPLIT and W.rel_fro(S, S_ref) < TOL_SPLIT
    # and the last chunk on its own
    assert W.rel_fro(o[-64:], o_ref[-64:]) < TOL_SPLIT


def test_prefill_config2_shape_reduced_heads(ctx):
    """BASELINE config 2's sequence length (T=32768, 512 chunks in one scan) at 2 heads."""
    rng = np.random.default_rng(0)
    T, H, d = 32768, 2, 128
    t = W.kda_tokens(rng, T, H, d, d, bf16=True)
    cu = np.array([0, T], np.int32)
    o, S = run_prefill(ctx, t["q"], t["k"], t["v"], t["g"], t["beta"], cu)
    o_ref, S_ref = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu,
                                         nthreads=oracle.max_threads())
    assert W.rel_fro(o, o_ref) < TOL_BF16
    assert W.rel_fro(S, S_ref) < TOL_BF16
