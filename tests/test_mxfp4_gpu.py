"""MXFP4 expert projections on the B200 (k3cuda_mxfp4_dequant, k3cuda_matmul_mxfp4,
k3cuda_matmul_mxfp4_batch) against the reference's checkpoint fixture and the oracle. Up to
four activation rows take the streaming kernel, anything else the bf16 GEMM path.

Dequantisation is exact, so it is compared bit for bit. The matmul sums in fp32 where the
reference sums in double: relative Frobenius error 1e-6 on the streaming path and 2e-5 on
the GEMM path (activations as bf16 hi + lo halves, 2^-16 of each element).
"""
import numpy as np
import pytest

import k3cuda
import workloads as W
from oracle import oracle

pytestmark = pytest.mark.gpu


def _matmul(ctx, x, packed, scales, group=32):
    T, n_in = x.shape
    rows = packed.shape[0]
    y = ctx.empty((T, rows), np.float32)
    n = ctx.matmul_mxfp4_workspace(T, n_in, rows, group)
    ws = ctx.empty((max(n, 1),), np.uint8)
    dx, dp, ds = ctx.upload(x), ctx.upload(packed), ctx.upload(scales)
    ctx.matmul_mxfp4(y, dx, dp, ds, n_in, rows, T, group, ws, n)
    return y.numpy()


def test_dequant_bit_exact_on_checkpoint_bytes(ctx, golden):
    d = golden("mxfp4")
    rows, n_in = d["expected"].shape
    dp, ds = ctx.upload(d["packed"]), ctx.upload(d["scales"])
    out = ctx.empty((rows, n_in), np.float32)
    ctx.mxfp4_dequant(out, dp, ds, rows, n_in, int(d["group"]))
    assert np.array_equal(out.numpy().view(np.uint32), d["expected"].view(np.uint32))
    outb = ctx.empty((rows, n_in), np.uint16)
    ctx.mxfp4_dequant(outb, dp, ds, rows, n_in, int(d["group"]), out_dtype=k3cuda.BF16)
    assert np.array_equal(W.bf16_to_f32(outb.numpy()).view(np.uint32),
                          d["expected"].view(np.uint32))  # every value is exact in bf16


@pytest.mark.parametrize("T", [1, 2])
def test_matmul_on_checkpoint_bytes_matches_reference(ctx, golden, T):
    """The streaming path on the real expert rows against the reference's own
    k3_matmul_mxfp4 output (stored with the fixture)."""
    d = golden("mxfp4")
    y = _matmul(ctx, d["x"][:T], d["packed"], d["scales"])
    assert W.rel_fro(y, d["y_ref"][:T]) < 1e-6


@pytest.mark.parametrize("T,rows,n_in,group,tol", [
    (1, 3072, 3584, 32, 1e-6),    # an expert's w1 / w3 at the model's shape, decode
    (3, 3584, 3072, 32, 1e-6),    # w2, three tokens
    (4, 301, 1024, 32, 1e-6),     # rows not a multiple of the warp's 4
    (1, 1000, 3584, 32, 1e-6),    # many row groups, the last one partial
    (2, 45, 7168, 32, 1e-6),      # longer rows
    (9, 300, 1024, 32, 2e-5),     # GEMM path
    (2, 40, 96, 16, 2e-5),        # group 16: GEMM path
    (1, 33, 100, 32, 2e-5),       # partial last group: GEMM path
])
def test_matmul_matches_oracle(ctx, T, rows, n_in, group, tol):
    rng = np.random.default_rng(T * 1000 + rows)
    packed = rng.integers(0, 256, (rows, n_in // 2), dtype=np.uint8)
    ngrp = (n_in + group - 1) // group
    scales = rng.integers(118, 128, (rows, ngrp), dtype=np.uint8)
    scales[0, 0], scales[-1, -1] = 255, 0  # NaN byte read as 0, and the subnormal scale
    x = rng.standard_normal((T, n_in)).astype(np.float32)
    y = _matmul(ctx, x, packed, scales, group)
    assert W.rel_fro(y, oracle.matmul_mxfp4(x, packed, scales, group)) < tol


def test_batch_of_experts_matches_single_calls(ctx):
    """Eight experts' w1 and w3 on one z plus their w2 on eight different activations, one
    launch each, equal to the per-matrix oracle."""
    rng = np.random.default_rng(5)
    n, rows, n_in = 16, 512, 1024
    packed = [rng.integers(0, 256, (rows, n_in // 2), dtype=np.uint8) for _ in range(n)]
    scales = [rng.integers(118, 128, (rows, n_in // 32), dtype=np.uint8) for _ in range(n)]
    z = rng.standard_normal((1, n_in)).astype(np.float32)
    acts = [rng.standard_normal((1, n_in)).astype(np.float32) for _ in range(n)]
    dp = [ctx.upload(p) for p in packed]
    ds = [ctx.upload(s) for s in scales]
    dz = ctx.upload(z)
    da = [ctx.upload(a) for a in acts]
    ys = [ctx.empty((1, rows), np.float32) for _ in range(n)]
    ctx.matmul_mxfp4_batch(ys, [dz] * n, dp, ds, n_in, rows, 1)
    for i in range(n):
        assert W.rel_fro(ys[i].numpy(), oracle.matmul_mxfp4(z, packed[i], scales[i])) < 1e-6
    ctx.matmul_mxfp4_batch(ys, da, dp, ds, n_in, rows, 1)
    for i in range(n):
        assert W.rel_fro(ys[i].numpy(), oracle.matmul_mxfp4(acts[i], packed[i], scales[i])) < 1e-6


def test_rejects_odd_width_and_large_group(ctx):
    x, y = ctx.empty((1, 8), np.float32), ctx.empty((1, 4), np.float32)
    p, s = ctx.empty((4, 4), np.uint8), ctx.empty((4, 1), np.uint8)
    for n_in, group in ((7, 32), (8, 128)):
        with pytest.raises(k3cuda.K3CudaError) as e:
            ctx.matmul_mxfp4(y, x, p, s, n_in, 4, 1, group)
        assert e.value.code == k3cuda.ERR_ARG
