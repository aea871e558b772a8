"""The layer drop-ins with the reference's exact signatures: k3g_mla_cached for
k3_mla_cached (include/k3/k3.h:219-221) and k3g_kda_layer for k3_kda_layer (:468-469), with
the reference's K3Cfg / K3MlaW / K3KdaW layouts (k3cuda.Cfg and the weight structs).

Checked against the reference's own k3_mla_cached (compiled from its unmodified sources,
oracle/_ref) over calls that carry the cache, and against its mla fixture:
  * any head geometry runs the fp32 path: held to the reference's own elementwise bar
    (MANIFEST: 1e-5 absolute + 1e-4 relative) on the fixture, 1e-4 relative Frobenius over
    carried calls;
  * the released geometry runs the bf16 tensor-core path: 5e-3 relative Frobenius.
Also: the cache resumes from a copy of its host rows, the one-token mode is bit-identical
however a sequence is cut into calls, and a position past the cache aborts the process with
the reference's message.
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

import k3cuda
import workloads as W
from oracle import oracle

pytestmark = pytest.mark.gpu
fp = C.POINTER(C.c_float)
HERE = os.path.dirname(os.path.abspath(__file__))


def P(a):
    return None if a is None else a.ctypes.data_as(fp)


class MlaW(C.Structure):
    """k3g_mla_weights: K3MlaW's layout (include/k3/k3.h:203-210)."""
    _fields_ = [(n, C.c_void_p) for n in ("q_a", "q_b", "kv_a", "kv_b", "o", "g", "q_a_norm",
                                          "kv_a_norm")] + [("wdt", C.c_int)]


def _mla_struct(w, wdt):
    proj = ("q_a", "q_b", "kv_a", "kv_b", "o", "g")
    keep, ptr = {}, {}
    for n in MlaW._fields_[:-1]:
        n = n[0]
        a = w.get(n)
        if a is None:
            ptr[n] = None
            continue
        a = np.ascontiguousarray(W.f32_to_bf16(a) if (wdt == 1 and n in proj) else a,
                                 np.uint16 if (wdt == 1 and n in proj) else np.float32)
        keep[n] = a
        ptr[n] = a.ctypes.data
    return MlaW(**ptr, wdt=wdt), keep


def _cfg(E, H, QL, dn, dr, dl, dv, eps=1e-5):
    return k3cuda.Cfg(hidden=E, n_heads=H, q_lora=QL, kv_lora=dl, qk_nope=dn, qk_rope=dr,
                      v_head=dv, rms_eps=eps, mla_out_gate=1)


def _fixture_weights(golden):
    d = golden("mla")
    w = dict(q_a=d["q_a_proj_weight"], q_b=d["q_b_proj_weight"],
             kv_a=d["kv_a_proj_with_mqa_weight"], kv_b=d["kv_b_proj_weight"],
             o=d["o_proj_weight"], g=d["g_proj_weight"], q_a_norm=d["q_a_layernorm_weight"],
             kv_a_norm=d["kv_a_layernorm_weight"])
    geo = dict(E=int(d["in"].shape[2]), H=int(d["n_heads"]), QL=int(d["q_lora"]),
               dn=int(d["qk_nope"]), dr=int(d["qk_rope"]), dl=int(d["kv_lora"]),
               dv=int(d["v_head"]))
    return d, w, geo


def test_mla_dropin_uncached_on_reference_fixture(golden):
    """k3_mla (k3_mla_cached without a cache) on the reference's mla fixture, whose geometry
    (24/8/32/16) takes the fp32 path: the reference's elementwise tolerance."""
    G = k3cuda.gpu_lib()
    G.k3g_shutdown()
    d, w, g = _fixture_weights(golden)
    ws, keep = _mla_struct(w, 0)
    c = _cfg(g["E"], g["H"], g["QL"], g["dn"], g["dr"], g["dl"], g["dv"], float(d["rms_eps"]))
    x = np.ascontiguousarray(d["in"][0], np.float32)
    T = x.shape[0]
    out = np.zeros_like(x)
    G.k3g_mla_cached(P(out), P(x), C.byref(ws), C.byref(c), T, None, None, None, 0, 0)
    tol = np.load(os.path.join(HERE, "golden", "manifest_tolerance.npz"))
    want = d["out"][0]
    assert np.all(np.abs(out - want) <= float(tol["fp32_abs"]) + float(tol["fp32_rel"]) *
                  np.abs(want)), np.max(np.abs(out - want))


def _carried(golden_w, g, wdt, seq, seed, copy_at=None):
    """Drive the drop-in and the compiled reference over calls of `seq` tokens carrying the
    cache; returns per-call relative errors (and, with copy_at, also continues on a copy of
    the host rows after that call and checks it gives the same outputs)."""
    G = k3cuda.gpu_lib()
    rng = np.random.default_rng(seed)
    ws, keep = _mla_struct(golden_w, wdt)
    c = _cfg(g["E"], g["H"], g["QL"], g["dn"], g["dr"], g["dl"], g["dv"])
    cap = sum(seq) + 3
    kvw = g["H"] * (g["dn"] + g["dv"])
    kvc, ropec = np.zeros((cap, kvw), np.float32), np.zeros((cap, g["dr"]), np.float32)
    rkvc, rropec = np.zeros_like(kvc), np.zeros_like(ropec)
    hostw = {n: (W.f32_to_bf16(a) if (wdt == 1 and n in ("q_a", "q_b", "kv_a", "kv_b", "o", "g")
                                       and a is not None) else a) for n, a in golden_w.items()}
    errs, cached = [], 0
    copies = None
    for i, T in enumerate(seq):
        x = rng.standard_normal((T, g["E"]), dtype=np.float32)
        want = oracle.ref_mla_cached(x, hostw, g["H"], g["QL"], 1e-5, rkvc, rropec, cached,
                                     wdt=wdt, kv_lora=g["dl"], qk_nope=g["dn"], qk_rope=g["dr"],
                                     v_head=g["dv"])
        out = np.zeros((T, g["E"]), np.float32)
        G.k3g_mla_cached(P(out), P(x), C.byref(ws), C.byref(c), T, None, P(kvc), P(ropec),
                         cached, cap)
        errs.append(W.rel_fro(out, want))
        if copies is not None:
            out2 = np.zeros_like(out)
            G.k3g_mla_cached(P(out2), P(x), C.byref(ws), C.byref(c), T, None, P(copies[0]),
                             P(copies[1]), cached, cap)
            assert np.array_equal(out2, out), i
        cached += T
        if copy_at == i:
            copies = (kvc.copy(), ropec.copy())
    return errs


def test_mla_dropin_carried_cache_any_geometry(golden):
    """The fixture's geometry over prefill / decode / chunk calls: fp32 path, 1e-4."""
    k3cuda.gpu_lib().k3g_shutdown()
    _, w, g = _fixture_weights(golden)
    errs = _carried(w, g, 0, (7, 1, 1, 3, 9, 1), 5)
    assert max(errs) < 1e-4, errs


@pytest.mark.parametrize("wdt", [0, 1])
def test_mla_dropin_carried_cache_released_geometry(wdt):
    """128/64/512/128 heads (the tensor-core path, bf16 cache) vs the reference, 5e-3; the
    cache continued from a copy of its host rows gives the same bytes."""
    k3cuda.gpu_lib().k3g_shutdown()
    rng = np.random.default_rng(3 + wdt)
    E, H, QL = 256, 2, 64
    f = lambda *s, sc=1.0: rng.standard_normal(s, dtype=np.float32) * np.float32(sc)  # noqa: E731
    w = dict(q_a=f(QL, E, sc=0.06), q_b=f(H * 192, QL, sc=0.12), kv_a=f(576, E, sc=0.06),
             kv_b=f(H * 256, 512, sc=0.04), o=f(E, H * 128, sc=0.08), g=f(H * 128, E, sc=0.06),
             q_a_norm=(1 + 0.1 * f(QL)).astype(np.float32),
             kv_a_norm=(1 + 0.1 * f(512)).astype(np.float32))
    g = dict(E=E, H=H, QL=QL, dn=128, dr=64, dl=512, dv=128)
    errs = _carried(w, g, wdt, (40, 1, 1, 5, 12, 1), 9, copy_at=2)
    assert max(errs) < 5e-3, errs


def test_mla_dropin_fp32_path_forced_at_released_geometry():
    """K3G_MLA_F32=1 takes the fp32 path at the released geometry: 1e-4 vs the reference."""
    G = k3cuda.gpu_lib()
    G.k3g_shutdown()
    rng = np.random.default_rng(21)
    E, H, QL = 256, 2, 64
    f = lambda *s, sc=1.0: rng.standard_normal(s, dtype=np.float32) * np.float32(sc)  # noqa: E731
    w = dict(q_a=f(QL, E, sc=0.06), q_b=f(H * 192, QL, sc=0.12), kv_a=f(576, E, sc=0.06),
             kv_b=f(H * 256, 512, sc=0.04), o=f(E, H * 128, sc=0.08), g=None,
             q_a_norm=(1 + 0.1 * f(QL)).astype(np.float32),
             kv_a_norm=(1 + 0.1 * f(512)).astype(np.float32))
    g = dict(E=E, H=H, QL=QL, dn=128, dr=64, dl=512, dv=128)
    os.environ["K3G_MLA_F32"] = "1"
    try:
        errs = _carried(w, g, 0, (20, 1, 4, 1), 4)
    finally:
        del os.environ["K3G_MLA_F32"]
        G.k3g_shutdown()
    assert max(errs) < 1e-4, errs


def test_tokenwise_mode_is_independent_of_chunking(golden):
    """K3G_TOKENWISE=1: a 9-token call equals nine 1-token calls bit for bit, for the MLA
    drop-in (cache rows too) and the KDA drop-in (state too)."""
    G = k3cuda.gpu_lib()
    G.k3g_shutdown()
    _, w, g = _fixture_weights(golden)
    ws, keep = _mla_struct(w, 0)
    c = _cfg(g["E"], g["H"], g["QL"], g["dn"], g["dr"], g["dl"], g["dv"])
    rng = np.random.default_rng(8)
    x = rng.standard_normal((9, g["E"]), dtype=np.float32)
    kvw = g["H"] * (g["dn"] + g["dv"])
    os.environ["K3G_TOKENWISE"] = "1"
    try:
        k1, r1 = np.zeros((12, kvw), np.float32), np.zeros((12, g["dr"]), np.float32)
        k2, r2 = k1.copy(), r1.copy()
        o1 = np.zeros_like(x)
        G.k3g_mla_cached(P(o1), P(x), C.byref(ws), C.byref(c), 9, None, P(k1), P(r1), 0, 12)
        o2 = np.zeros_like(x)
        for t in range(9):
            xt, ot = np.ascontiguousarray(x[t:t + 1]), np.zeros((1, g["E"]), np.float32)
            G.k3g_mla_cached(P(ot), P(xt), C.byref(ws), C.byref(c), 1, None, P(k2), P(r2), t, 12)
            o2[t] = ot[0]
        assert np.array_equal(o1, o2) and np.array_equal(k1, k2) and np.array_equal(r1, r2)
        # KDA
        d = golden("kda_layer8")
        E, H, D, K = d["in"].shape[2], int(d["H"]), int(d["d_k"]), int(d["conv_k"])
        kw = {}
        keepk = []
        for kn, on in zip(k3cuda.KDA_WEIGHT_NAMES, oracle.LAYER_WEIGHTS):
            a = np.ascontiguousarray(d[on], np.float32)
            keepk.append(a)
            kw[kn] = a.ctypes.data
        kws = k3cuda.KdaWeights(**kw, wdt=0)
        kc = k3cuda.Cfg(hidden=E, kda_heads=H, kda_head_dim=D, conv_k=K, gate_lb=-5.0,
                        rms_eps=1e-5)
        xs = rng.standard_normal((9, E)).astype(np.float32)
        s1 = np.zeros(H * D * D + 3 * H * D * (K - 1), np.float32)
        s2 = s1.copy()
        y1 = np.zeros_like(xs)
        G.k3g_kda_layer(P(y1), P(xs), C.byref(kws), C.byref(kc), 9, P(s1), None)
        y2 = np.zeros_like(xs)
        for t in range(9):
            xt, yt = np.ascontiguousarray(xs[t:t + 1]), np.zeros((1, E), np.float32)
            G.k3g_kda_layer(P(yt), P(xt), C.byref(kws), C.byref(kc), 1, P(s2), None)
            y2[t] = yt[0]
        assert np.array_equal(y1, y2) and np.array_equal(s1, s2)
    finally:
        del os.environ["K3G_TOKENWISE"]
        G.k3g_shutdown()


def test_mla_dropin_aborts_past_the_cache():
    """A position at or past cap aborts the process with the reference's message (the check
    runs on the host before any device work)."""
    code = f"""
import ctypes as C, sys
sys.path[:0] = [{os.path.dirname(HERE)!r}, {os.path.join(os.path.dirname(HERE), 'kimi-k3-in-c_b200')!r}]
import numpy as np, k3cuda
G = k3cuda.gpu_lib()
c = k3cuda.Cfg(hidden=128, n_heads=4, q_lora=64, kv_lora=32, qk_nope=24, qk_rope=8, v_head=16,
               rms_eps=1e-5)
kvc = np.zeros((8, 160), np.float32); ropec = np.zeros((8, 8), np.float32)
x = np.zeros((4, 128), np.float32); out = np.zeros_like(x)
fp = C.POINTER(C.c_float)
G.k3g_mla_cached(out.ctypes.data_as(fp), x.ctypes.data_as(fp), None, C.byref(c), 4, None,
                 kvc.ctypes.data_as(fp), ropec.ctypes.data_as(fp), 6, 8)
"""
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode != 0
    assert "MLA KV cache position is 9, which exceeds the limit of 7" in r.stderr
