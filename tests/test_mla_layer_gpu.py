"""The MLA layer forward on the device (k3cuda_mla_layer) against the reference's own
k3_mla_cached (compiled from its sources, oracle/_ref) over a sequence of calls that carry
the cache: a 70-token prefill (GEMM projections), single decode tokens, a 5-token chunk
(streaming projections). The device keeps the latent cache, the reference its expanded
keys and values; each call's output must agree within the 5e-3 relative Frobenius bar for
bf16 attention operands, with fp32 and bf16 weights, with and without the output gate."""
import numpy as np
import pytest

import k3cuda
import workloads as W
from oracle import oracle

pytestmark = pytest.mark.gpu

E, H, QL, CAP = 256, 2, 64, 128


def _weights(rng, gate):
    f = lambda *s, sc=1.0: rng.standard_normal(s, dtype=np.float32) * np.float32(sc)  # noqa: E731
    w = dict(q_a=f(QL, E, sc=0.06), q_b=f(H * 192, QL, sc=0.12), kv_a=f(576, E, sc=0.06),
             kv_b=f(H * 256, 512, sc=0.04), o=f(E, H * 128, sc=0.08),
             g=f(H * 128, E, sc=0.06) if gate else None,
             q_a_norm=(1 + 0.1 * f(QL)).astype(np.float32),
             kv_a_norm=(1 + 0.1 * f(512)).astype(np.float32))
    return w


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("wdt,gate", [(0, True), (1, True), (1, False)])
def test_mla_layer_matches_reference_over_calls(ctx, wdt, gate):
    rng = np.random.default_rng(11 + 2 * wdt + gate)
    w = _weights(rng, gate)
    proj = ("q_a", "q_b", "kv_a", "kv_b", "o", "g")
    host = {n: (W.f32_to_bf16(a) if (wdt == 1 and n in proj and a is not None) else a)
            for n, a in w.items()}
    dev = {n: (ctx.upload(a) if a is not None else None) for n, a in host.items()}
    latent = ctx.empty((CAP, 512), np.uint16)
    rope = ctx.empty((CAP, 64), np.uint16)
    kvc = np.zeros((CAP, H * 256), np.float32)
    ropec = np.zeros((CAP, 64), np.float32)
    cached = 0
    for T in (70, 1, 1, 5, 1):
        x = rng.standard_normal((T, E), dtype=np.float32)
        want = oracle.ref_mla_cached(x, host, H, QL, 1e-5, kvc, ropec, cached, wdt=wdt)
        out = ctx.empty((T, E), np.float32)
        n = ctx.mla_layer_workspace(T, E, H, QL, cached, wdt)
        ws = ctx.empty((n,), np.uint8)
        xb = ctx.upload(x)
        ctx.mla_layer(out, xb, dev, wdt, T, E, H, QL, 1e-5, latent, rope, cached, CAP, ws, n)
        got = out.numpy()
        assert W.rel_fro(got, want) < 5e-3, (T, cached, W.rel_fro(got, want))
        cached += T


def test_mla_layer_refuses_past_the_cache(ctx):
    rng = np.random.default_rng(1)
    w = _weights(rng, True)
    dev = {n: ctx.upload(a) for n, a in w.items()}
    latent, rope = ctx.empty((8, 512), np.uint16), ctx.empty((8, 64), np.uint16)
    out, x = ctx.empty((4, E), np.float32), ctx.empty((4, E), np.float32)
    with pytest.raises(k3cuda.K3CudaError) as e:
        ctx.mla_layer(out, x, dev, 0, 4, E, H, QL, 1e-5, latent, rope, 6, 8, None, 0)
    assert e.value.code == k3cuda.ERR_ARG
