"""The allocation-free prefill entry point, k3cuda_kda_prefill_noalloc (GPU).

It serves callers that cannot allocate device memory where they run a prefill (a host
runtime that owns the whole HBM budget through its own allocator, or a latency-critical
path that cannot afford cudaMalloc's implicit synchronisation): its workspace is a static
device array inside libk3cuda instead of a caller buffer. It must give the same results as
k3cuda_kda_prefill with a caller workspace, call after call, since every call reuses the
array and finds the previous call's contents in it.

This file sorts last so that a run stopping at the first failure has already run the rest.
"""
import numpy as np
import pytest

import k3cuda
import workloads as W

pytestmark = pytest.mark.gpu

TOL_BF16 = 5e-3   # bf16 outputs, as the prefill parity tests
TOL_F32 = 2e-3    # fp32 state


def _inputs(seed):
    rng = np.random.default_rng(seed)
    H, d = 4, 128
    cu = np.array([0, 100, 100, 300], np.int32)  # includes an empty sequence
    t = W.kda_tokens(rng, int(cu[-1]), H, d, d, bf16=True)
    S0 = rng.standard_normal((3, H, d, d), dtype=np.float32) * np.float32(0.05)
    return t, cu, S0, H, d


def _upload(ctx, t, S0):
    bf = W.f32_to_bf16
    return (ctx.upload(S0), ctx.upload(bf(t["q"])), ctx.upload(bf(t["k"])), ctx.upload(bf(t["v"])),
            ctx.upload(t["g"]), ctx.upload(t["beta"]))


def test_noalloc_matches_workspace_entry_point_twice(ctx):
    t, cu, S0, H, d = _inputs(31)
    T = int(cu[-1])
    qs = 1.0 / np.sqrt(np.float32(d))

    # the existing entry point, with a caller-allocated workspace
    dS, dq, dk, dv, dg, db = _upload(ctx, t, S0)
    do = ctx.empty((T, H, d), np.uint16)
    nws = ctx.kda_prefill_workspace(cu, H, d, d)
    ws = ctx.empty((nws,), np.uint8)
    ctx.kda_prefill(dS, do, dq, dk, dv, dg, db, cu, H, d, d, qs, ws, nws)
    o_ref = W.bf16_to_f32(do.numpy())
    S_ref = dS.numpy()

    # the allocation-free entry point, two calls in a row on fresh copies of the state
    for call in range(2):
        dS2 = ctx.upload(S0)
        do2 = ctx.empty((T, H, d), np.uint16)
        ctx.kda_prefill_noalloc(dS2, do2, dq, dk, dv, dg, db, cu, H, d, d, qs)
        o = W.bf16_to_f32(do2.numpy())
        S = dS2.numpy()
        assert W.rel_fro(o, o_ref) < TOL_BF16, call
        assert W.rel_fro(S, S_ref) < TOL_F32, call
        assert np.array_equal(S[1], S0[1]), call  # the empty sequence keeps its state


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    cu = np.array([0, 32768], np.int32)
    H, d = 32, 128
    assert ctx.kda_prefill_workspace(cu, H, d, d) > (64 << 20)
    with pytest.raises(k3cuda.K3CudaError) as ei:
        ctx.kda_prefill_noalloc(None, None, None, None, None, None, None, cu, H, d, d, 0.088)
    assert ei.value.code == k3cuda.ERR_WORKSPACE
    assert "static scratch" in str(ei.value)
