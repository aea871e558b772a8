"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE, not product code).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` / ``--impl
reference`` legs import this module, and only to check or to time the reference. The
product library (libk3cuda) never calls into it.

Two libraries:
  * ``liboracle.so``      -- our C restatement (oracle/k3_oracle.c), each function citing
                             the reference file:line it follows;
  * ``_ref/libk3ref.so``  -- the reference's unmodified src/core/k3_ops.c compiled by
                             oracle/Makefile, plus loops in ref_driver.c.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def lib():
    """Load (building if needed) the restatement library."""
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.orc_kda_step.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, C.c_float, C.c_int, C.c_int]
        L.orc_kda_recurrence.argtypes = [C.c_void_p, f32p, f32p, f32p, f32p, f32p, C.c_int, f32p,
                                         i32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                         C.c_int]
        L.orc_kda_decay.argtypes = [f32p, f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_float]
        L.orc_kda_layer.argtypes = ([f32p, f32p] + [C.c_int] * 5 + [C.c_float, C.c_float]
                                    + [f32p] * 14 + [C.c_void_p])
        L.orc_mla_absorbed_decode.argtypes = ([f32p] * 7 + [i32p] + [C.c_int] * 7
                                              + [C.c_float, C.c_int])
        L.orc_kda_chunked_f64.argtypes = [f32p, f32p, f64p, f64p, f32p, f32p, f32p, f32p, f32p,
                                          C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
        L.orc_mxfp4_dequant.argtypes = [f32p, u8p, u8p, C.c_int, C.c_int, C.c_int]
        L.orc_matmul_mxfp4.argtypes = [f32p, f32p, u8p, u8p, C.c_int, C.c_int, C.c_int, C.c_int]
        _LIB = L
    return _LIB


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libk3ref.so"))


def ref():
    """Load the compiled reference (oracle/_ref/libk3ref.so)."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libk3ref.so")
        if not os.path.exists(path):
            build()
        R = C.CDLL(path)
        R.k3_kda_step.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, C.c_float, C.c_int, C.c_int]
        R.k3ref_kda_recurrence.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, C.c_int, f32p,
                                           i32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                           C.c_int]
        R.k3ref_kda_decode.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, C.c_int, f32p,
                                       C.c_long, C.c_int, C.c_int, C.c_float, C.c_int]
        R.k3ref_max_threads.restype = C.c_int
        R.k3_kda_decay.argtypes = [f32p, f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_float]
        R.k3_rmsnorm.argtypes = [f32p, f32p, f32p, C.c_int, C.c_float]
        R.k3_matmul.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int]
        R.k3_mla_scratch_cached.restype = C.c_size_t
        u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
        R.k3_mxfp4_dequant.argtypes = [f32p, u8p, u8p, C.c_int, C.c_int, C.c_int]
        R.k3_matmul_mxfp4.argtypes = [f32p, f32p, u8p, u8p, C.c_int, C.c_int, C.c_int]
        R.k3ref_mla_cached.argtypes = ([f32p, f32p] + [C.c_int] * 8 + [C.c_float]
                                       + [C.c_void_p] * 6 + [f32p, f32p, C.c_int, f32p, f32p,
                                                             C.c_int, C.c_int])
        R.k3ref_kda_layer.argtypes = ([f32p, f32p] + [C.c_int] * 5 + [C.c_float, C.c_float]
                                      + [C.c_void_p] * 3 + [f32p] * 3 + [C.c_void_p] * 2
                                      + [f32p] * 2 + [C.c_void_p] * 2 + [f32p, C.c_void_p,
                                                                         C.c_int, C.c_void_p])
        _REF = R
    return _REF


def build():
    """Compile liboracle.so and, where the reference sources exist, _ref/libk3ref.so."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE], check=True)


# ----------------------------------------------------------------------------- KDA
def kda_recurrence(q, k, v, gate, beta, cu_seqlens, *, gate_is_log=True, q_scale=None,
                   state=None, nthreads=1, use_ref=False):
    """Packed varlen KDA recurrence. q,k [sumT,H,dk]; v [sumT,H,dv]; gate [sumT,H,dk];
    beta [sumT,H]; cu_seqlens int32 [nseq+1]. Returns (o [sumT,H,dv], S [nseq,H,dk,dv]).
    ``use_ref`` runs the reference's own k3_kda_step instead of the restatement."""
    q, k, v, gate, beta = (_f32(a) for a in (q, k, v, gate, beta))
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
    T, H, dk = q.shape
    dv = v.shape[2]
    nseq = len(cu) - 1
    if q_scale is None:
        q_scale = 1.0 / float(np.sqrt(np.float32(dk)))
    S = (np.zeros((nseq, H, dk, dv), np.float32) if state is None
         else np.array(state, dtype=np.float32, copy=True, order="C"))
    o = np.zeros((T, H, dv), np.float32)
    if use_ref:
        ref().k3ref_kda_recurrence(S, o, q, k, v, gate, int(gate_is_log), beta, cu, nseq, H, dk,
                                   dv, float(q_scale), int(nthreads))
    else:
        lib().orc_kda_recurrence(S.ctypes.data, o, q, k, v, gate, int(gate_is_log), beta, cu,
                                 nseq, H, dk, dv, float(q_scale), int(nthreads))
    return o, S


def kda_decode(S, q, k, v, gate, beta, *, gate_is_log=True, q_scale=None, nthreads=1,
               use_ref=False):
    """One decode token for B sequences: S [B,H,dk,dv] (copied, not modified);
    q,k [B,H,dk], v [B,H,dv], gate [B,H,dk], beta [B,H]. Returns (o [B,H,dv], S_new)."""
    B, H, dk = q.shape
    dv = v.shape[2]
    if q_scale is None:
        q_scale = 1.0 / float(np.sqrt(np.float32(dk)))
    if use_ref:
        S2 = np.array(S, dtype=np.float32, copy=True, order="C")
        o = np.zeros((B, H, dv), np.float32)
        ref().k3ref_kda_decode(S2, o, _f32(q), _f32(k), _f32(v), _f32(gate), int(gate_is_log),
                               _f32(beta), B * H, dk, dv, float(q_scale), int(nthreads))
        return o, S2
    cu = np.arange(B + 1, dtype=np.int32)
    o, S2 = kda_recurrence(q.reshape(B, H, dk), k, v, gate, beta, cu, gate_is_log=gate_is_log,
                           q_scale=q_scale, state=S, nthreads=nthreads)
    return o, S2


def kda_chunked_f64(q, k, v, g, beta, C, q_scale):
    """Chunkwise double-precision restatement for one head: q,k,g [T,dk], v [T,dv], beta [T].
    Returns (o, S, Akk, Aqk)."""
    q, k, v, g, beta = (_f32(a) for a in (q, k, v, g, beta))
    T, dk = q.shape
    dv = v.shape[1]
    n = T // C
    o = np.zeros((T, dv), np.float32)
    S = np.zeros((dk, dv), np.float32)
    Akk = np.zeros((n, C, C), np.float64)
    Aqk = np.zeros((n, C, C), np.float64)
    lib().orc_kda_chunked_f64(o, S, Akk, Aqk, q, k, v, g, beta, T, C, dk, dv, float(q_scale))
    return o, S, Akk, Aqk


# ----------------------------------------------------------------------------- MLA
def mla_absorbed_decode(q_nope, q_rope, latent, rope, w_uk, w_uv, ctx_lens, scale,
                        nthreads=1):
    """q_nope [B,H,dn], q_rope [B,H,dr], latent [B,cap,dl], rope [B,cap,dr],
    w_uk [H,dn,dl], w_uv [H,dv,dl], ctx_lens int32 [B]. Returns out [B,H,dv] fp32."""
    q_nope, q_rope, latent, rope, w_uk, w_uv = (_f32(a) for a in
                                               (q_nope, q_rope, latent, rope, w_uk, w_uv))
    B, H, dn = q_nope.shape
    dr = q_rope.shape[2]
    cap, dl = latent.shape[1], latent.shape[2]
    dv = w_uv.shape[1]
    out = np.zeros((B, H, dv), np.float32)
    cl = np.ascontiguousarray(ctx_lens, dtype=np.int32)
    lib().orc_mla_absorbed_decode(out, q_nope, q_rope, latent, rope, w_uk, w_uv, cl, B, cap, H,
                                  dn, dr, dl, dv, float(scale), int(nthreads))
    return out


# ------------------------------------------------------------------------ KDA layer
# Weight names as the reference's layer fixtures store them (tests/golden/kda_layer*.npz),
# in the argument order of orc_kda_layer / K3KdaW.
LAYER_WEIGHTS = ("q_proj", "k_proj", "v_proj", "q_conv", "k_conv", "v_conv", "f_a", "f_b",
                 "A_log", "dt_bias", "b_proj", "g_proj", "o_norm", "o_proj")
LAYER_PROJ = ("q_proj", "k_proj", "v_proj", "f_a", "f_b", "b_proj", "g_proj", "o_proj")


def kda_layer(x, w, H, D, K, lb, eps, state=None):
    """orc_kda_layer (restatement of k3_kda_layer, src/core/k3_ops.c:864-951) on x [T][E]
    with fp32 weights `w` (LAYER_WEIGHTS). state: flat fp32 [H*D*D + 3*H*D*(K-1)], updated
    in place, or None."""
    x = _f32(x)
    T, E = x.shape
    out = np.zeros((T, E), np.float32)
    args = [_f32(w[n]) for n in LAYER_WEIGHTS]
    lib().orc_kda_layer(out, x, T, E, H, D, K, float(lb), float(eps), *args,
                        None if state is None else state.ctypes.data)
    return out


def ref_kda_layer(x, w, H, D, K, lb, eps, state=None, wdt=0):
    """The reference's own k3_kda_layer (oracle/_ref). wdt 1: the projection weights in `w`
    are bf16 bit patterns (uint16), as the real checkpoint stores them."""
    x = _f32(x)
    T, E = x.shape
    out = np.zeros((T, E), np.float32)
    keep, args = [], []
    for n in LAYER_WEIGHTS:
        if n in LAYER_PROJ:
            a = np.ascontiguousarray(w[n], np.uint16 if wdt == 1 else np.float32)
            keep.append(a)
            args.append(a.ctypes.data)
        else:
            args.append(_f32(w[n]))
    ref().k3ref_kda_layer(out, x, T, E, H, D, K, float(lb), float(eps), *args, int(wdt),
                          None if state is None else state.ctypes.data)
    return out


# ------------------------------------------------------------------------ MLA layer
MLA_WEIGHTS = ("q_a", "q_b", "kv_a", "kv_b", "o", "g", "q_a_norm", "kv_a_norm")


def ref_mla_cached(x, w, H, q_lora, eps, kvc, ropec, cached, wdt=0, kv_lora=512, qk_nope=128,
                   qk_rope=64, v_head=128):
    """The reference's own k3_mla_cached (oracle/_ref) on x [T][E] with its EXPANDED caches
    kvc [cap][H*(qk_nope+v_head)] and ropec [cap][qk_rope] (updated in place). w: host
    weights by MLA_WEIGHTS name (projections fp32, or bf16 bits when wdt=1; "g" may be
    None)."""
    x = _f32(x)
    T, E = x.shape
    out = np.zeros((T, E), np.float32)
    keep, ptrs = [], []
    for n in ("q_a", "q_b", "kv_a", "kv_b", "o", "g"):
        if w.get(n) is None:
            ptrs.append(None)
            continue
        a = np.ascontiguousarray(w[n], np.uint16 if wdt == 1 else np.float32)
        keep.append(a)
        ptrs.append(a.ctypes.data)
    cap = kvc.shape[0]
    ref().k3ref_mla_cached(out, x, T, E, H, q_lora, kv_lora, qk_nope, qk_rope, v_head,
                           float(eps), *ptrs, _f32(w["q_a_norm"]), _f32(w["kv_a_norm"]),
                           int(wdt), kvc, ropec, int(cached), int(cap))
    return out


# --------------------------------------------------------------------------- MXFP4
def mxfp4_dequant(packed, scales, group=32):
    """orc_mxfp4_dequant: packed uint8 [rows][in/2], scales uint8 [rows][in/group]."""
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.uint8)
    rows, in_ = packed.shape[0], 2 * packed.shape[1]
    out = np.zeros((rows, in_), np.float32)
    lib().orc_mxfp4_dequant(out, packed, scales, rows, in_, group)
    return out


def matmul_mxfp4(x, packed, scales, group=32, use_ref=False):
    """y [T][rows] = x [T][in] W^T with W as MXFP4: the restatement (double products and
    sums), or with use_ref the reference's own k3_matmul_mxfp4 once per row of x."""
    x = _f32(np.atleast_2d(x))
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.uint8)
    T, in_ = x.shape
    rows = packed.shape[0]
    y = np.zeros((T, rows), np.float32)
    if use_ref:
        for t in range(T):
            yt = np.zeros(rows, np.float32)
            ref().k3_matmul_mxfp4(yt, np.ascontiguousarray(x[t]), packed, scales, in_, rows,
                                  group)
            y[t] = yt
    else:
        lib().orc_matmul_mxfp4(y, x, packed, scales, in_, rows, T, group)
    return y


def max_threads() -> int:
    return os.cpu_count() or 1
