"""The allocation-free prefill entry point, k3cuda_kda_prefill_noalloc (GPU).

It serves callers that cannot allocate device memory where they run a prefill (a host
runtime that owns the whole HBM budget through its own allocator, or a latency-critical
path that cannot afford cudaMalloc's implicit synchronisation): its workspace is a static
device array inside libk3cuda instead of a caller buffer. It must give the same results as
k3cuda_kda_prefill with a caller workspace, call after call, since every call reuses the
array and finds the previous call's contents in it.

The two entry points run the same kernels on the same inputs, so their outputs must agree
byte for byte. To show that no kernel reads a scratch byte it has not written first, the
shared array is dirtied by an unrelated call (other lengths, heads and values) before the
checked calls, and the reference run gets a caller workspace filled with 0xFF.

This file sorts last so that a run stopping at the first failure has already run the rest.
"""
import numpy as np
import pytest

import k3cuda
import workloads as W

pytestmark = pytest.mark.gpu

TOL_BF16 = 5e-3   # bf16 outputs against the oracle, as the prefill parity tests
TOL_F32 = 2e-3    # fp32 outputs and state against the oracle


def _case(seed, cu, H, d, bf16):
    rng = np.random.default_rng(seed)
    cu = np.asarray(cu, np.int32)
    t = W.kda_tokens(rng, int(cu[-1]), H, d, d, bf16=bf16)
    S0 = rng.standard_normal((len(cu) - 1, H, d, d), dtype=np.float32) * np.float32(0.05)
    return t, cu, S0


def _upload(ctx, t, S0, bf16):
    cv = W.f32_to_bf16 if bf16 else (lambda a: a)
    return (ctx.upload(S0), ctx.upload(cv(t["q"])), ctx.upload(cv(t["k"])),
            ctx.upload(cv(t["v"])), ctx.upload(t["g"]), ctx.upload(t["beta"]))


def _dirty_scratch(ctx, seed):
    """One no-alloc call on an unrelated batch: several long sequences at d=128, bf16, so the
    static array holds bytes of another shape when the checked calls run."""
    t, cu, S0 = _case(seed, [0, 700, 1500, 1501, 2600], 8, 128, True)
    dS, dq, dk, dv, dg, db = _upload(ctx, t, S0, True)
    do = ctx.empty((int(cu[-1]), 8, 128), np.uint16)
    ctx.kda_prefill_noalloc(dS, do, dq, dk, dv, dg, db, cu, 8, 128, 128, 0.07)
    ctx.sync()


# (lengths, heads, head width, bf16 I/O): the tensor-core path (bf16, d=128) and the
# CUDA-core paths (fp32 I/O; d=64), each with partial chunks and an empty sequence
CASES = [
    ([0, 100, 100, 300], 4, 128, True),
    ([0, 36, 36, 44, 300], 3, 128, False),
    ([0, 8, 129, 129, 230], 5, 64, True),
]


@pytest.mark.parametrize("cu,H,d,bf16", CASES)
def test_noalloc_matches_workspace_entry_point_twice(ctx, cu, H, d, bf16):
    from oracle import oracle

    t, cu, S0 = _case(31 + H, cu, H, d, bf16)
    T = int(cu[-1])
    qs = 1.0 / np.sqrt(np.float32(d))
    odt = np.uint16 if bf16 else np.float32
    io = k3cuda.BF16 if bf16 else k3cuda.F32

    # the existing entry point, with a caller-allocated workspace full of 0xFF bytes
    dS, dq, dk, dv, dg, db = _upload(ctx, t, S0, bf16)
    do = ctx.empty((T, H, d), odt)
    nws = ctx.kda_prefill_workspace(cu, H, d, d)
    ws = ctx.empty((nws,), np.uint8)
    ws.fill(0xFF)
    ctx.kda_prefill(dS, do, dq, dk, dv, dg, db, cu, H, d, d, qs, ws, nws, io_dtype=io)
    o_ref = do.numpy()
    S_ref = dS.numpy()

    # sanity: that run is the recurrence (the oracle, on the same rounded inputs)
    o_orc, S_orc = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu,
                                         state=S0, nthreads=8)
    o_f = W.bf16_to_f32(o_ref) if bf16 else o_ref
    assert W.rel_fro(o_f, o_orc) < (TOL_BF16 if bf16 else TOL_F32)
    assert W.rel_fro(S_ref, S_orc) < (TOL_BF16 if bf16 else TOL_F32)

    # the allocation-free entry point, two calls in a row on fresh copies of the state,
    # after an unrelated call has left its bytes in the shared array
    _dirty_scratch(ctx, 7 + H)
    for call in range(2):
        dS2 = ctx.upload(S0)
        do2 = ctx.empty((T, H, d), odt)
        ctx.kda_prefill_noalloc(dS2, do2, dq, dk, dv, dg, db, cu, H, d, d, qs, io_dtype=io)
        o = do2.numpy()
        S = dS2.numpy()
        assert np.array_equal(o, o_ref), call
        assert np.array_equal(S, S_ref), call
        empty = [i for i in range(len(cu) - 1) if cu[i] == cu[i + 1]]
        for i in empty:
            assert np.array_equal(S[i], S0[i]), call  # an empty sequence keeps its state


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    cu = np.array([0, 32768], np.int32)
    H, d = 32, 128
    assert ctx.kda_prefill_workspace(cu, H, d, d) > k3cuda.NOALLOC_SCRATCH_BYTES
    with pytest.raises(k3cuda.K3CudaError) as ei:
        ctx.kda_prefill_noalloc(None, None, None, None, None, None, None, cu, H, d, d, 0.088)
    assert ei.value.code == k3cuda.ERR_WORKSPACE
    assert "static scratch" in str(ei.value)
