"""The KDA layer forward on the device (k3cuda_kda_layer) and its projection primitive
(k3cuda_matmul) against the CPU oracle.

The oracle's orc_kda_layer is bit-identical to the reference's own k3_kda_layer (pinned in
test_oracle.py) and reproduces the reference's layer fixtures. Tolerances are relative
Frobenius errors: 2e-3 with fp32 recurrence operands and 5e-3 with bf16 ones, the bounds
the attention path is held to; the projections alone are held to 2e-5.
"""
import numpy as np
import pytest

import workloads as W
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = {0: 2e-3, 1: 5e-3}  # by recurrence io dtype (F32, BF16)


def _weights_to_device(ctx, w, wdt):
    """Upload fixture-named fp32 weights; projections as bf16 when wdt is BF16. Returns the
    device mapping (k3cuda names) and the fp32 weights the oracle must use (bf16 widened)."""
    import k3cuda
    dev, used = {}, {}
    names = dict(zip(k3cuda.KDA_WEIGHT_NAMES, oracle.LAYER_WEIGHTS))
    for kn, on in names.items():
        a = np.ascontiguousarray(w[on], np.float32)
        if on in oracle.LAYER_PROJ and wdt == k3cuda.BF16:
            bits = W.f32_to_bf16(a)
            dev[kn] = ctx.upload(bits)
            used[on] = W.bf16_to_f32(bits)
        else:
            dev[kn] = ctx.upload(a.reshape(a.shape[0], -1) if a.ndim == 3 else a)
            used[on] = a
    return dev, used


def _run_layer(ctx, dev, wdt, x, H, D, K, lb, eps, state, io):
    T, E = x.shape
    out = ctx.empty((T, E), np.float32)
    n = ctx.kda_layer_workspace(T, E, H, D, K, wdt, io)
    ws = ctx.empty((max(n, 1),), np.uint8)
    xb = ctx.upload(np.ascontiguousarray(x, np.float32))
    ctx.kda_layer(out, xb, dev, wdt, T, E, H, D, K, lb, eps, state, io, ws, n)
    return out.numpy()


@pytest.mark.parametrize("wdt", [0, 1])
@pytest.mark.parametrize("T,n_in,n_out", [(1, 128, 96), (2, 1024, 300), (8, 7168, 130),
                                          (9, 256, 96), (40, 1024, 300), (128, 64, 256),
                                          (129, 7168, 700), (300, 1536, 40), (1000, 512, 1031),
                                          (33, 16, 64), (77, 200, 99)])
def test_matmul_matches_double(ctx, wdt, T, n_in, n_out):
    """y = x W^T for the matvec kernel (T <= 8) and the GEMMs (T > 8: tcgen05 over x's bf16
    hi/lo halves for bf16 weights with in % 64 == 0, the CUDA-core kernel for fp32 weights
    and other widths), fp32 and bf16 weights, partial token and row tiles, against float64."""
    import k3cuda
    rng = np.random.default_rng(T * 7 + n_out + wdt)
    x = rng.standard_normal((T, n_in)).astype(np.float32)
    Wt = (rng.standard_normal((n_out, n_in)) / np.sqrt(n_in)).astype(np.float32)
    if wdt == k3cuda.BF16:
        bits = W.f32_to_bf16(Wt)
        Wt, dW = W.bf16_to_f32(bits), ctx.upload(bits)
    else:
        dW = ctx.upload(Wt)
    y = ctx.empty((T, n_out), np.float32)
    n = ctx.matmul_workspace(T, n_in, wdt)
    ws = ctx.empty((max(n, 1),), np.uint8)
    xb = ctx.upload(x)
    ctx.matmul(y, xb, dW, wdt, n_in, n_out, T, ws, n)
    want = x.astype(np.float64) @ Wt.astype(np.float64).T
    assert W.rel_fro(y.numpy(), want) < 2e-5


def test_matmul_refuses_unaligned_width(ctx):
    import k3cuda
    x, Wt, y = ctx.empty((1, 12), np.float32), ctx.empty((4, 12), np.float32), ctx.empty((1, 4),
                                                                                          np.float32)
    with pytest.raises(k3cuda.K3CudaError) as e:
        ctx.matmul(y, x, Wt, k3cuda.F32, 12, 4, 1)
    assert e.value.code == k3cuda.ERR_UNSUPPORTED


@pytest.mark.parametrize("name", ["kda_layer1", "kda_layer8"])
def test_layer_matches_reference_fixture(ctx, golden, name):
    """The reference's own layer fixtures (fp32 weights, fresh state, D = 16: the per-token
    decode path): output and final recurrent state; a NULL state gives the same output."""
    import k3cuda
    d = golden(name)
    T, E = d["in"].shape[1], d["in"].shape[2]
    H, D, K = int(d["H"]), int(d["d_k"]), int(d["conv_k"])
    dev, _ = _weights_to_device(ctx, d, k3cuda.F32)
    S = ctx.upload(np.zeros(H * D * D + 3 * H * D * (K - 1), np.float32))
    out = _run_layer(ctx, dev, k3cuda.F32, d["in"][0], H, D, K, float(d["lower_bound"]),
                     float(d["rms_eps"]), S, k3cuda.F32)
    assert W.rel_fro(out, d["out"][0]) < TOL[0]
    assert W.rel_fro(S.numpy()[: H * D * D], d["state_out"].ravel()) < TOL[0]
    out0 = _run_layer(ctx, dev, k3cuda.F32, d["in"][0], H, D, K, float(d["lower_bound"]),
                      float(d["rms_eps"]), None, k3cuda.F32)
    assert np.array_equal(out0, out)


@pytest.mark.parametrize("io", [0, 1])
@pytest.mark.parametrize("wdt", [0, 1])
def test_layer_carried_state_matches_oracle(ctx, wdt, io):
    """D = 128 over a sequence of calls carrying the state (recurrent and conv history):
    prefill lengths on the GEMM path (70, 130, 9), decode (1), and calls shorter than the
    conv history (1, 2) on the matvec path; every output and the final state."""
    rng = np.random.default_rng(60 + 2 * wdt + io)
    E, H, D, K = 256, 2, 128, 4
    w = W.kda_layer_weights(rng, E, H, D, K)
    dev, used = _weights_to_device(ctx, w, wdt)
    s0 = (0.1 * rng.standard_normal(H * D * D + 3 * H * D * (K - 1))).astype(np.float32)
    s_orc, S = s0.copy(), ctx.upload(s0)
    for T in (70, 1, 2, 9, 5, 130, 1):
        x = rng.standard_normal((T, E)).astype(np.float32)
        want = oracle.kda_layer(x, used, H, D, K, -5.0, 1e-5, s_orc)
        got = _run_layer(ctx, dev, wdt, x, H, D, K, -5.0, 1e-5, S, io)
        assert W.rel_fro(got, want) < TOL[io], T
    got_s = S.numpy()
    assert W.rel_fro(got_s[: H * D * D], s_orc[: H * D * D]) < TOL[io]
    # the conv history is the raw projections of the last K-1 tokens: fp32 either way
    assert W.rel_fro(got_s[H * D * D:], s_orc[H * D * D:]) < 2e-5


@pytest.mark.parametrize("D,T", [(64, 33), (32, 12)])
def test_layer_other_head_dims(ctx, D, T):
    """D = 64 (chunked prefill, SIMT form) and D = 32 (decode once per token), fp32."""
    import k3cuda
    rng = np.random.default_rng(D + T)
    E, H, K = 192, 3, 4
    w = W.kda_layer_weights(rng, E, H, D, K)
    dev, used = _weights_to_device(ctx, w, k3cuda.F32)
    s_orc = np.zeros(H * D * D + 3 * H * D * (K - 1), np.float32)
    S = ctx.upload(s_orc)
    for t in (T, 1):
        x = rng.standard_normal((t, E)).astype(np.float32)
        want = oracle.kda_layer(x, used, H, D, K, -5.0, 1e-5, s_orc)
        got = _run_layer(ctx, dev, k3cuda.F32, x, H, D, K, -5.0, 1e-5, S, k3cuda.F32)
        assert W.rel_fro(got, want) < TOL[0], t
    assert W.rel_fro(S.numpy(), s_orc) < TOL[0]


def test_layer_model_width(ctx):
    """The model's hidden width E = 7168 with bf16 weights (4 heads of 128): decode and a
    16-token prefill on the tensor-core recurrence."""
    import k3cuda
    rng = np.random.default_rng(7)
    E, H, D, K = 7168, 4, 128, 4
    w = W.kda_layer_weights(rng, E, H, D, K)
    dev, used = _weights_to_device(ctx, w, k3cuda.BF16)
    s_orc = np.zeros(H * D * D + 3 * H * D * (K - 1), np.float32)
    S = ctx.upload(s_orc)
    for T in (16, 1):
        x = rng.standard_normal((T, E)).astype(np.float32)
        want = oracle.kda_layer(x, used, H, D, K, -5.0, 1e-5, s_orc)
        got = _run_layer(ctx, dev, k3cuda.BF16, x, H, D, K, -5.0, 1e-5, S, k3cuda.BF16)
        assert W.rel_fro(got, want) < TOL[1], T
