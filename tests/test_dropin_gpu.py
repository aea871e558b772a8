"""The C99 drop-ins (include/k3_gpu.h) with the reference's own signatures and fixtures.

These are the calls a reference caller switches to: host fp32 buffers, the reference's
argument order, abort-on-failure. They are checked on the reference's fixtures exactly as
the reference's tests/unit/test_ops.c drives k3_kda_step (t_recur, :310-350).
"""
import ctypes as C
import os

import numpy as np
import pytest

import k3cuda
import workloads as W

pytestmark = pytest.mark.gpu
fp = C.POINTER(C.c_float)
W_GOLDEN_TOL = os.path.join(os.path.dirname(__file__), "golden", "manifest_tolerance.npz")


def P(a):
    return a.ctypes.data_as(fp)


@pytest.mark.parametrize("name", ["kda_recur1", "kda_recur8"])
def test_kda_step_dropin_on_reference_fixture(golden, name):
    G = k3cuda.gpu_lib()
    d = golden(name)
    T, H, dk = d["q"].shape
    qs = np.float32(d["q_scale"])
    S = np.zeros((H, dk, dk), np.float32)
    out = np.zeros((T, H, dk), np.float32)
    for t in range(T):
        for h in range(H):
            q = np.ascontiguousarray(d["q"][t, h] * qs)
            o = np.zeros(dk, np.float32)
            Sh = np.ascontiguousarray(S[h])
            G.k3g_kda_step(P(Sh), P(o), P(q), P(np.ascontiguousarray(d["k"][t, h])),
                           P(np.ascontiguousarray(d["v"][t, h])),
                           P(np.ascontiguousarray(d["alpha"][t, h])), float(d["beta"][t, h]), dk, dk)
            S[h] = Sh
            out[t, h] = o
    assert W.rel_fro(out, d["out"]) < 1e-5 and W.rel_fro(S, d["state_out"]) < 1e-5


def test_kda_recurrence_dropin_config0(golden):
    """k3_kda_layer's recurrence block (k3_ops.c:908-938) on config 0 through the drop-in:
    alpha in, q scaled inside, state carried in place; 256 prefill then 32 single steps."""
    G = k3cuda.gpu_lib()
    d = golden("cfg0_kda")
    T, H, D = d["q"].shape
    alpha = np.exp(d["g"]).astype(np.float32)
    S = np.zeros((H, D, D), np.float32)
    out = np.zeros((T, H, D), np.float32)
    f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
    o = np.zeros((256, H, D), np.float32)
    G.k3g_kda_recurrence(P(S), P(o), P(f(d["q"][:256])), P(f(d["k"][:256])), P(f(d["v"][:256])),
                         P(f(alpha[:256])), P(f(d["beta"][:256])), 256, H, D)
    out[:256] = o
    for t in range(256, T):
        o1 = np.zeros((1, H, D), np.float32)
        G.k3g_kda_recurrence(P(S), P(o1), P(f(d["q"][t:t + 1])), P(f(d["k"][t:t + 1])),
                             P(f(d["v"][t:t + 1])), P(f(alpha[t:t + 1])),
                             P(f(d["beta"][t:t + 1])), 1, H, D)
        out[t] = o1[0]
    assert W.rel_fro(out, d["out"]) < 2e-3 and W.rel_fro(S, d["state_out"]) < 2e-3


def test_mla_attend_dropin_on_reference_output(golden):
    """kv_b in the reference's layout; the drop-in splits W_UK/W_UV itself."""
    G = k3cuda.gpu_lib()
    m = golden("mla_ref_full")
    Pn = m["q_nope"].shape[0]
    H, qn = m["q_nope"].shape[1:]
    qr = m["q_rope"].shape[2]
    dl = m["latent"].shape[2]
    vh = m["w_uv"].shape[1]
    kv_b = np.ascontiguousarray(np.concatenate([m["w_uk"], m["w_uv"]], axis=1).reshape(-1, dl))
    scale = float(m["scale"].ravel()[0])
    for p in (1, 17, 64, Pn):
        q = np.ascontiguousarray(np.concatenate([m["q_nope"][p - 1], m["q_rope"][p - 1]], axis=1))
        acc = np.zeros((H, vh), np.float32)
        G.k3g_mla_attend(P(acc), P(q), P(np.ascontiguousarray(m["latent"][0, :p])),
                         P(np.ascontiguousarray(m["rope"][0, :p])), P(kv_b), scale, H, qn, qr, dl,
                         vh, p)
        assert W.rel_fro(acc, m["out"][p - 1]) < 5e-3, p


def _host_weights(w, wdt):
    """k3g_kda_weights over host arrays (fixture names), projections as bf16 bits when wdt=1.
    Returns the struct, the arrays it points into (kept alive), and the fp32 weights the
    oracle must use."""
    from oracle import oracle
    keep, used, ptrs = [], {}, {}
    for kn, on in zip(k3cuda.KDA_WEIGHT_NAMES, oracle.LAYER_WEIGHTS):
        a = np.ascontiguousarray(w[on], np.float32)
        if on in oracle.LAYER_PROJ and wdt == 1:
            bits = W.f32_to_bf16(a)
            keep.append(bits)
            used[on] = W.bf16_to_f32(bits)
            ptrs[kn] = bits.ctypes.data
        else:
            keep.append(a)
            used[on] = a
            ptrs[kn] = a.ctypes.data
    return k3cuda.KdaWeights(**ptrs, wdt=wdt), keep, used


@pytest.mark.parametrize("name", ["kda_layer1", "kda_layer8"])
def test_kda_layer_dropin_on_reference_fixture(golden, name):
    """k3g_kda_layer with the reference fixture's K3KdaW-ordered host weights: output and the
    final recurrent state, as tests/unit/test_ops.c checks k3_kda_layer."""
    G = k3cuda.gpu_lib()
    G.k3g_shutdown()  # the weight cache is keyed by host address: start from an empty one
    d = golden(name)
    T, E = d["in"].shape[1], d["in"].shape[2]
    H, D, K = int(d["H"]), int(d["d_k"]), int(d["conv_k"])
    w, keep, _ = _host_weights(d, 0)
    x = np.ascontiguousarray(d["in"][0], np.float32)
    out = np.zeros((T, E), np.float32)
    state = np.zeros(H * D * D + 3 * H * D * (K - 1), np.float32)
    c = k3cuda.Cfg(hidden=E, kda_heads=H, kda_head_dim=D, conv_k=K,
                   gate_lb=float(d["lower_bound"]), rms_eps=float(d["rms_eps"]))
    scratch = np.zeros(16, np.float32)  # accepted, not touched
    G.k3g_kda_layer(P(out), P(x), C.byref(w), C.byref(c), T, P(state), P(scratch))
    G.k3g_shutdown()
    assert W.rel_fro(out, d["out"][0]) < 2e-3
    assert W.rel_fro(state[: H * D * D], d["state_out"].ravel()) < 2e-3
    # and at the reference's own elementwise bar (its MANIFEST: atol + rtol * |want|)
    tol = np.load(W_GOLDEN_TOL)
    lim = float(tol["fp32_abs"]) + float(tol["fp32_rel"]) * np.abs(d["out"][0])
    assert np.all(np.abs(out - d["out"][0]) <= lim)


def test_kda_layer_dropin_bf16_weights_decode_loop():
    """bf16 weights (the real checkpoint's type), D = 128: a 12-token prefill then four
    decode calls carrying the host state, against the oracle step by step."""
    from oracle import oracle
    G = k3cuda.gpu_lib()
    G.k3g_shutdown()
    rng = np.random.default_rng(77)
    E, H, D, K = 256, 2, 128, 4
    w, keep, used = _host_weights(W.kda_layer_weights(rng, E, H, D, K), 1)
    s_gpu = (0.1 * rng.standard_normal(H * D * D + 3 * H * D * (K - 1))).astype(np.float32)
    s_orc = s_gpu.copy()
    c = k3cuda.Cfg(hidden=E, kda_heads=H, kda_head_dim=D, conv_k=K, gate_lb=-5.0,
                   rms_eps=1e-5)
    for T in (12, 1, 1, 1, 1):
        x = rng.standard_normal((T, E)).astype(np.float32)
        out = np.zeros((T, E), np.float32)
        G.k3g_kda_layer(P(out), P(x), C.byref(w), C.byref(c), T, P(s_gpu), None)
        want = oracle.kda_layer(x, used, H, D, K, -5.0, 1e-5, s_orc)
        assert W.rel_fro(out, want) < 2e-3, T
    G.k3g_shutdown()
    assert W.rel_fro(s_gpu, s_orc) < 2e-3
