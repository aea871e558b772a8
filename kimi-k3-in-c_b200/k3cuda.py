"""ctypes binding of libk3cuda (include/k3cuda.h) and the C99 drop-in libk3gpu (include/k3_gpu.h).

This is the Python side of the C ABI, used by the tests, ``bench.py`` and
``__graft_entry__``. It adds no arithmetic: every call goes straight to the CUDA library
and raises ``K3CudaError`` with the library's message when the status is not zero. There
is no CPU fallback -- if ``libk3cuda.so`` is missing or no B200 is visible, loading fails
loudly.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libk3cuda.so")
GPU_LIB_PATH = os.path.join(HERE, "libk3gpu.so")

OK, ERR_ARG, ERR_CUDA, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_NCCL, ERR_TIMEOUT, ERR_STATE = range(8)
F32, BF16 = 0, 1
GATE_LOG, GATE_ALPHA = 0, 1
MAX_EVENTS = 64
NOALLOC_SCRATCH_BYTES = 64 << 20   # K3CUDA_NOALLOC_SCRATCH_BYTES

# Every symbol include/k3cuda.h declares, with (restype, argtypes).
_vp, _i, _f, _sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
_ip = C.POINTER(C.c_int)
SIGNATURES = {
    "k3cuda_init": (_i, [_i, C.POINTER(_vp)]),
    "k3cuda_shutdown": (_i, [_vp]),
    "k3cuda_last_error": (C.c_char_p, []),
    "k3cuda_device_count": (_i, [_ip]),
    "k3cuda_sync": (_i, [_vp]),
    "k3cuda_stream": (_vp, [_vp]),
    "k3cuda_set_wait_limit": (_i, [_vp, C.c_longlong]),
    "k3cuda_wait_selftest": (_i, [_vp]),
    "k3cuda_malloc": (_i, [_vp, C.POINTER(_vp), _sz]),
    "k3cuda_free": (_i, [_vp, _vp]),
    "k3cuda_host_alloc": (_i, [_vp, C.POINTER(_vp), _sz]),
    "k3cuda_host_free": (_i, [_vp, _vp]),
    "k3cuda_memcpy_h2d": (_i, [_vp, _vp, _vp, _sz]),
    "k3cuda_memcpy_d2h": (_i, [_vp, _vp, _vp, _sz]),
    "k3cuda_memcpy_d2d": (_i, [_vp, _vp, _vp, _sz]),
    "k3cuda_memset": (_i, [_vp, _vp, _i, _sz]),
    "k3cuda_event_record": (_i, [_vp, _i]),
    "k3cuda_event_elapsed": (_i, [_vp, _i, _i, C.POINTER(_f)]),
    "k3cuda_launch_count": (C.c_longlong, [_vp]),
    "k3cuda_flush_l2": (_i, [_vp]),
    "k3cuda_kda_decode": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _i,
                               _i]),
    "k3cuda_kda_decode_host_workspace": (_i, [_i, _i, _i, _i, _i, C.POINTER(_sz)]),
    "k3cuda_kda_decode_host": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f,
                                    _i, _i, _i, _vp, _sz]),
    "k3cuda_kda_prefill_workspace": (_i, [_ip, _i, _i, _i, _i, _i, C.POINTER(_sz)]),
    "k3cuda_kda_prefill": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _ip, _i, _i, _i, _i, _f,
                                _i, _i, _i, _vp, _sz]),
    "k3cuda_kda_prefill_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _ip, _i, _i, _i,
                                        _i, _f, _i, _i, _i]),
    "k3cuda_mla_decode_workspace": (_i, [_ip, _i, _i, _i, _i, C.POINTER(_sz)]),
    "k3cuda_mla_plan_stats": (_i, [_ip, _i, _i, _ip, _ip, C.POINTER(_sz)]),
    "k3cuda_mla_decode": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _ip, _i, _i, _i, _i,
                               _i, _i, _i, _f, _vp, _sz]),
    "k3cuda_mla_attend": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _ip, _ip, _i, _i, _i,
                               _i, _i, _i, _i, _i, _f, _vp, _sz]),
    "k3cuda_mla_cache_append": (_i, [_vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _i, _i, _i]),
    "k3cuda_mla_layer_workspace": (_i, [_i, _i, _i, _i, _i, _i, C.POINTER(_sz)]),
    "k3cuda_mla_layer": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp,
                              _i, _i, _vp, _sz]),
    "k3cuda_mla_layer_f32_workspace": (_i, [_i, _i, _i, _i, _i, _i, _i, _i, _i,
                                            C.POINTER(_sz)]),
    "k3cuda_mla_layer_f32": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp,
                                  _vp, _i, _i, _vp, _sz]),
    "k3cuda_comm_unique_id": (_i, [C.c_char_p]),
    "k3cuda_comm_init": (_i, [_vp, _i, _i, C.c_char_p]),
    "k3cuda_comm_set_timeout": (_i, [_vp, _i]),
    "k3cuda_allgather_heads_workspace": (_i, [_i, _i, _i, _i, _i, C.POINTER(_sz)]),
    "k3cuda_allgather_heads": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz]),
    "k3cuda_comm_register_full": (_i, [_vp, _vp, _sz]),
    "k3cuda_kda_prefill_gathered": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _ip, _i, _i, _i, _i,
                                         _f, _i, _i, _vp, _sz]),
    "k3cuda_matmul_workspace": (_i, [_i, _i, _i, C.POINTER(_sz)]),
    "k3cuda_matmul": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz]),
    "k3cuda_mxfp4_dequant": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i, _i]),
    "k3cuda_matmul_mxfp4_workspace": (_i, [_i, _i, _i, _i, C.POINTER(_sz)]),
    "k3cuda_matmul_mxfp4": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz]),
    "k3cuda_matmul_mxfp4_batch": (_i, [_vp, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp),
                                       C.POINTER(_vp), _i, _i, _i, _i]),
    "k3cuda_kda_layer_workspace": (_i, [_i, _i, _i, _i, _i, _i, _i, C.POINTER(_sz)]),
    "k3cuda_kda_layer": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _f, _vp, _i, _vp, _sz]),
}


class KdaWeights(C.Structure):
    """k3cuda_kda_weights: device pointers of one KDA layer, in K3KdaW's field order."""
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("q_conv", _vp), ("k_conv", _vp),
                ("v_conv", _vp), ("f_a", _vp), ("f_b", _vp), ("A_log", _vp), ("dt_bias", _vp),
                ("b", _vp), ("g", _vp), ("o_norm", _vp), ("o", _vp), ("wdt", _i)]


class MlaWeights(C.Structure):
    """k3cuda_mla_weights: device pointers of one MLA layer, in K3MlaW's field order."""
    _fields_ = [("q_a", _vp), ("q_b", _vp), ("kv_a", _vp), ("kv_b", _vp), ("o", _vp),
                ("g", _vp), ("q_a_norm", _vp), ("kv_a_norm", _vp), ("wdt", _i)]


class Cfg(C.Structure):
    """k3g_cfg: field for field the reference's K3Cfg (include/k3/k3.h:73-120)."""
    _fields_ = [("hidden", _i), ("n_layers", _i), ("vocab", _i), ("rms_eps", _f),
                ("kda_heads", _i), ("kda_head_dim", _i), ("conv_k", _i), ("gate_lb", _f),
                ("n_heads", _i), ("q_lora", _i), ("kv_lora", _i), ("qk_nope", _i),
                ("qk_rope", _i), ("v_head", _i), ("mla_out_gate", _i), ("n_experts", _i),
                ("topk", _i), ("n_shared", _i), ("latent", _i), ("moe_inter", _i),
                ("routed_scale", _f), ("moe_renorm", _i), ("latent_norm", _i),
                ("first_dense", _i), ("dense_inter", _i), ("attn_res_block", _i),
                ("situ_b1", _f), ("situ_b2", _f), ("n_full_attn", _i),
                ("full_attn", C.POINTER(_i))]


KDA_WEIGHT_NAMES = ("q", "k", "v", "q_conv", "k_conv", "v_conv", "f_a", "f_b", "A_log",
                    "dt_bias", "b", "g", "o_norm", "o")

# include/k3_gpu.h: the reference-signature C99 wrappers (host fp32 buffers).
_fp = C.POINTER(C.c_float)
GPU_SIGNATURES = {
    "k3g_kda_step": (None, [_fp, _fp, _fp, _fp, _fp, _fp, _f, _i, _i]),
    "k3g_kda_recurrence": (None, [_fp, _fp, _fp, _fp, _fp, _fp, _fp, _i, _i, _i]),
    "k3g_mla_attend": (None, [_fp, _fp, _fp, _fp, _fp, _f, _i, _i, _i, _i, _i, _i]),
    "k3g_kda_layer": (None, [_fp, _fp, _vp, _vp, _i, _fp, _fp]),
    "k3g_mla_cached": (None, [_fp, _fp, _vp, _vp, _i, _fp, _fp, _fp, _i, _i]),
    "k3g_mla_cache_forget": (None, [_fp]),
    "k3g_state_save": (_i, [C.c_char_p, _ip, _ip, _i, _vp, C.c_int64, _i, _vp, _vp, _i, _i, _i,
                            _i, _i]),
    "k3g_state_load": (_i, [C.c_char_p, _ip, _ip, _i, _ip, _vp, C.c_int64, _i, _vp, _vp, _i, _i,
                            _i, _i, _ip]),
    "k3g_shutdown": (None, []),
}


class K3CudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libk3cuda error {code}: {msg}")
        self.code = code


_lib = None
_gpu = None


def build(quiet: bool = True) -> None:
    """Compile libk3cuda.so and libk3gpu.so in place (nvcc cross-compiles without a GPU)."""
    cmd = ["make", "-j8", "-C", HERE]
    subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL if quiet else None)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing; run make -C {HERE}")
        L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def gpu_lib():
    global _gpu
    if _gpu is None:
        lib()
        G = C.CDLL(GPU_LIB_PATH)
        for name, (res, args) in GPU_SIGNATURES.items():
            fn = getattr(G, name)
            fn.restype = res
            fn.argtypes = args
        _gpu = G
    return _gpu


def check(rc: int) -> None:
    if rc != OK:
        raise K3CudaError(rc, lib().k3cuda_last_error().decode(errors="replace"))


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, DeviceBuffer):
        return x.ptr
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    return int(x)


def _iarr(a):
    a = np.ascontiguousarray(a, dtype=np.int32)
    return a, a.ctypes.data_as(_ip)


class Context:
    """One libk3cuda context (device + stream)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().k3cuda_init(int(device), C.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            lib().k3cuda_shutdown(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # memory ----------------------------------------------------------------------
    def empty(self, shape, dtype) -> "DeviceBuffer":
        return DeviceBuffer(self, shape, dtype)

    def upload(self, arr: np.ndarray, dtype=None) -> "DeviceBuffer":
        arr = np.ascontiguousarray(arr if dtype is None else arr.astype(dtype))
        buf = DeviceBuffer(self, arr.shape, arr.dtype)
        buf.copy_from(arr)
        return buf

    def sync(self):
        check(lib().k3cuda_sync(self.h))

    def record(self, slot: int):
        check(lib().k3cuda_event_record(self.h, slot))

    def elapsed_ms(self, a: int, b: int) -> float:
        ms = C.c_float()
        check(lib().k3cuda_event_elapsed(self.h, a, b, C.byref(ms)))
        return float(ms.value)

    def launches(self) -> int:
        return int(lib().k3cuda_launch_count(self.h))

    def flush_l2(self):
        check(lib().k3cuda_flush_l2(self.h))

    def host_alloc(self, nbytes: int):
        p = C.c_void_p()
        check(lib().k3cuda_host_alloc(self.h, C.byref(p), int(nbytes)))
        return p.value

    def host_free(self, p):
        check(lib().k3cuda_host_free(self.h, p))

    def pinned(self, shape, dtype) -> np.ndarray:
        """numpy array over page-locked host memory (freed with the context's process)."""
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        p = self.host_alloc(max(n, 1))
        buf = (C.c_char * max(n, 1)).from_address(p)
        return np.frombuffer(buf, dtype=dtype, count=int(np.prod(shape))).reshape(shape)

    # hot path --------------------------------------------------------------------
    def kda_decode(self, state, o, q, k, v, gate, beta, n_streams, H, dk, dv, q_scale,
                   io_dtype=BF16, gate_mode=GATE_LOG):
        check(lib().k3cuda_kda_decode(self.h, _ptr(state), _ptr(o), _ptr(q), _ptr(k), _ptr(v),
                                      _ptr(gate), _ptr(beta), int(n_streams), int(H), int(dk),
                                      int(dv), float(q_scale), int(io_dtype), int(gate_mode)))

    def kda_decode_host_workspace(self, n_streams, H, dk, dv, io_dtype=BF16) -> int:
        n = C.c_size_t()
        check(lib().k3cuda_kda_decode_host_workspace(int(n_streams), int(H), int(dk), int(dv),
                                                     int(io_dtype), C.byref(n)))
        return int(n.value)

    def kda_decode_host(self, state, o, q, k, v, gate, beta, n_streams, H, dk, dv, q_scale,
                        staging, staging_bytes, io_dtype=BF16, gate_mode=GATE_LOG, slices=0):
        """k3cuda_kda_decode_host: o, q, k, v, gate, beta are host numpy arrays (C-contiguous,
        ideally from pinned()), state and staging device buffers. o is complete after sync()."""
        for a in (o, q, k, v, gate, beta):
            assert isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"]
        check(lib().k3cuda_kda_decode_host(self.h, _ptr(state), _ptr(o), _ptr(q), _ptr(k),
                                           _ptr(v), _ptr(gate), _ptr(beta), int(n_streams),
                                           int(H), int(dk), int(dv), float(q_scale),
                                           int(io_dtype), int(gate_mode), int(slices),
                                           _ptr(staging), int(staging_bytes)))

    def kda_prefill_workspace(self, cu_seqlens, H, dk, dv, chunk=64) -> int:
        cu, cup = _iarr(cu_seqlens)
        n = C.c_size_t()
        check(lib().k3cuda_kda_prefill_workspace(cup, len(cu) - 1, int(H), int(dk), int(dv),
                                                 int(chunk), C.byref(n)))
        return int(n.value)

    def kda_prefill(self, state, o, q, k, v, gate, beta, cu_seqlens, H, dk, dv, q_scale,
                    workspace, workspace_bytes, io_dtype=BF16, gate_mode=GATE_LOG, chunk=64):
        cu, cup = _iarr(cu_seqlens)
        check(lib().k3cuda_kda_prefill(self.h, _ptr(state), _ptr(o), _ptr(q), _ptr(k), _ptr(v),
                                       _ptr(gate), _ptr(beta), cup, len(cu) - 1, int(H),
                                       int(dk), int(dv), float(q_scale), int(io_dtype),
                                       int(gate_mode), int(chunk), _ptr(workspace),
                                       int(workspace_bytes)))

    def kda_prefill_noalloc(self, state, o, q, k, v, gate, beta, cu_seqlens, H, dk, dv, q_scale,
                            io_dtype=BF16, gate_mode=GATE_LOG, chunk=64):
        """k3cuda_kda_prefill with the library's static scratch instead of a workspace."""
        cu, cup = _iarr(cu_seqlens)
        check(lib().k3cuda_kda_prefill_noalloc(self.h, _ptr(state), _ptr(o), _ptr(q), _ptr(k),
                                               _ptr(v), _ptr(gate), _ptr(beta), cup, len(cu) - 1,
                                               int(H), int(dk), int(dv), float(q_scale),
                                               int(io_dtype), int(gate_mode), int(chunk)))

    def mla_decode_workspace(self, ctx_lens, H, dl=512, dv=128) -> int:
        cl, clp = _iarr(ctx_lens)
        n = C.c_size_t()
        check(lib().k3cuda_mla_decode_workspace(clp, len(cl), int(H), int(dl), int(dv),
                                                C.byref(n)))
        return int(n.value)

    def mla_decode(self, out, q_nope, q_rope, latent, rope, w_uk, w_uv, ctx_lens, cap, H,
                   scale, workspace, workspace_bytes, out_dtype=F32, dn=128, dr=64, dl=512,
                   dv=128):
        cl, clp = _iarr(ctx_lens)
        check(lib().k3cuda_mla_decode(self.h, _ptr(out), int(out_dtype), _ptr(q_nope),
                                      _ptr(q_rope), _ptr(latent), _ptr(rope), _ptr(w_uk),
                                      _ptr(w_uv), clp, len(cl), int(cap), int(H), int(dn),
                                      int(dr), int(dl), int(dv), float(scale), _ptr(workspace),
                                      int(workspace_bytes)))

    # projections and the KDA layer ------------------------------------------------
    def matmul_workspace(self, T, n_in, wdt) -> int:
        return _ws_query(lib().k3cuda_matmul_workspace, int(T), int(n_in), int(wdt))

    def matmul(self, y, x, W, wdt, n_in, n_out, T, workspace=None, workspace_bytes=0):
        check(lib().k3cuda_matmul(self.h, _ptr(y), _ptr(x), _ptr(W), int(wdt), int(n_in),
                                  int(n_out), int(T), _ptr(workspace), int(workspace_bytes)))

    def mxfp4_dequant(self, out, packed, scales, rows, n_in, group=32, out_dtype=F32):
        check(lib().k3cuda_mxfp4_dequant(self.h, _ptr(out), int(out_dtype), _ptr(packed),
                                         _ptr(scales), int(rows), int(n_in), int(group)))

    def matmul_mxfp4_workspace(self, T, n_in, rows, group=32) -> int:
        return _ws_query(lib().k3cuda_matmul_mxfp4_workspace, int(T), int(n_in), int(rows),
                         int(group))

    def matmul_mxfp4(self, y, x, packed, scales, n_in, rows, T, group=32, workspace=None,
                     workspace_bytes=0):
        check(lib().k3cuda_matmul_mxfp4(self.h, _ptr(y), _ptr(x), _ptr(packed), _ptr(scales),
                                        int(n_in), int(rows), int(group), int(T),
                                        _ptr(workspace), int(workspace_bytes)))

    def matmul_mxfp4_batch(self, ys, xs, packeds, scaless, n_in, rows, T):
        n = len(ys)
        arr = lambda bufs: (_vp * max(n, 1))(*[_ptr(b) for b in bufs])  # noqa: E731
        check(lib().k3cuda_matmul_mxfp4_batch(self.h, arr(ys), arr(xs), arr(packeds),
                                              arr(scaless), n, int(n_in), int(rows), int(T)))

    def kda_layer_workspace(self, T, E, H, D, K, wdt, io_dtype) -> int:
        return _ws_query(lib().k3cuda_kda_layer_workspace, int(T), int(E), int(H), int(D),
                         int(K), int(wdt), int(io_dtype))

    def kda_layer(self, out, x, weights, wdt, T, E, H, D, K, gate_lb, rms_eps, state,
                  io_dtype, workspace, workspace_bytes):
        """weights: mapping of KDA_WEIGHT_NAMES to device buffers (or device addresses)."""
        w = KdaWeights(**{n: _ptr(weights[n]) for n in KDA_WEIGHT_NAMES}, wdt=int(wdt))
        check(lib().k3cuda_kda_layer(self.h, _ptr(out), _ptr(x), C.byref(w), int(T), int(E),
                                     int(H), int(D), int(K), float(gate_lb), float(rms_eps),
                                     _ptr(state), int(io_dtype), _ptr(workspace),
                                     int(workspace_bytes)))

    def mla_attend(self, out, q_nope, q_rope, latent, rope, w_uk, w_uv, cache_seq, ctx_lens,
                   n_cache, cap, H, scale, workspace, workspace_bytes, out_dtype=F32):
        cs, csp = _iarr(cache_seq)
        cl, clp = _iarr(ctx_lens)
        check(lib().k3cuda_mla_attend(self.h, _ptr(out), int(out_dtype), _ptr(q_nope),
                                      _ptr(q_rope), _ptr(latent), _ptr(rope), _ptr(w_uk),
                                      _ptr(w_uv), csp, clp, len(cl), int(n_cache), int(cap),
                                      int(H), 128, 64, 512, 128, float(scale), _ptr(workspace),
                                      int(workspace_bytes)))

    def mla_cache_append(self, latent, rope, ct, kv_a_norm, eps, seq, pos0, T, n_cache, cap):
        check(lib().k3cuda_mla_cache_append(self.h, _ptr(latent), _ptr(rope), _ptr(ct),
                                            _ptr(kv_a_norm), float(eps), int(seq), int(pos0),
                                            int(T), int(n_cache), int(cap), 512, 64))

    def mla_layer_workspace(self, T, E, H, q_lora, cached, wdt) -> int:
        return _ws_query(lib().k3cuda_mla_layer_workspace, int(T), int(E), int(H), int(q_lora),
                         int(cached), int(wdt))

    def mla_layer(self, out, x, weights, wdt, T, E, H, q_lora, rms_eps, latent, rope, cached,
                  cap, workspace, workspace_bytes):
        """weights: mapping of MlaWeights field names to device buffers ("g" may be None)."""
        w = MlaWeights(**{n: _ptr(weights.get(n)) for n, _ in MlaWeights._fields_[:-1]},
                       wdt=int(wdt))
        check(lib().k3cuda_mla_layer(self.h, _ptr(out), _ptr(x), C.byref(w), int(T), int(E),
                                     int(H), int(q_lora), 128, 64, 512, 128, float(rms_eps),
                                     _ptr(latent), _ptr(rope), int(cached), int(cap),
                                     _ptr(workspace), int(workspace_bytes)))

    def mla_layer_f32_workspace(self, T, E, H, q_lora, dn, dr, dl, dv, wdt) -> int:
        return _ws_query(lib().k3cuda_mla_layer_f32_workspace, int(T), int(E), int(H),
                         int(q_lora), int(dn), int(dr), int(dl), int(dv), int(wdt))

    def mla_layer_f32(self, out, x, weights, wdt, T, E, H, q_lora, dn, dr, dl, dv, rms_eps,
                      latent, rope, cached, cap, workspace, workspace_bytes):
        """Any head geometry, fp32 latent/rope cache (k3cuda_mla_layer_f32)."""
        w = MlaWeights(**{n: _ptr(weights.get(n)) for n, _ in MlaWeights._fields_[:-1]},
                       wdt=int(wdt))
        check(lib().k3cuda_mla_layer_f32(self.h, _ptr(out), _ptr(x), C.byref(w), int(T), int(E),
                                         int(H), int(q_lora), int(dn), int(dr), int(dl), int(dv),
                                         float(rms_eps), _ptr(latent), _ptr(rope), int(cached),
                                         int(cap), _ptr(workspace), int(workspace_bytes)))

    # multi-GPU -------------------------------------------------------------------
    def set_wait_limit(self, cycles: int):
        check(lib().k3cuda_set_wait_limit(self.h, int(cycles)))

    def wait_selftest(self):
        check(lib().k3cuda_wait_selftest(self.h))

    def comm_set_timeout(self, ms: int):
        check(lib().k3cuda_comm_set_timeout(self.h, int(ms)))

    def comm_init(self, nranks: int, rank: int, uid: bytes):
        check(lib().k3cuda_comm_init(self.h, int(nranks), int(rank), uid))

    def allgather_heads_workspace(self, nranks, T, H_local, dv, dtype=BF16) -> int:
        n = C.c_size_t()
        check(lib().k3cuda_allgather_heads_workspace(int(nranks), int(T), int(H_local), int(dv),
                                                     int(dtype), C.byref(n)))
        return int(n.value)

    def allgather_heads(self, full, local, T, H_local, dv, workspace, workspace_bytes,
                        dtype=BF16):
        check(lib().k3cuda_allgather_heads(self.h, _ptr(full), _ptr(local), int(T), int(H_local),
                                           int(dv), int(dtype), _ptr(workspace),
                                           int(workspace_bytes)))

    def comm_register_full(self, full):
        """Map every rank's full-output buffer into every process (collective)."""
        check(lib().k3cuda_comm_register_full(self.h, _ptr(full), int(full.nbytes)))

    def kda_prefill_gathered(self, state, q, k, v, gate, beta, cu_seqlens, H_local, dk, dv,
                             q_scale, workspace, workspace_bytes, gate_mode=GATE_LOG, chunk=64):
        """Head-sharded prefill writing into every rank's registered full buffer (collective)."""
        cu, cup = _iarr(cu_seqlens)
        check(lib().k3cuda_kda_prefill_gathered(self.h, _ptr(state), _ptr(q), _ptr(k), _ptr(v),
                                                _ptr(gate), _ptr(beta), cup, len(cu) - 1,
                                                int(H_local), int(dk), int(dv), float(q_scale),
                                                int(gate_mode), int(chunk), _ptr(workspace),
                                                int(workspace_bytes)))


def _ws_query(fn, *args) -> int:
    n = C.c_size_t()
    check(fn(*args, C.byref(n)))
    return int(n.value)


def comm_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().k3cuda_comm_unique_id(buf))
    return buf.raw


def device_count() -> int:
    n = C.c_int()
    check(lib().k3cuda_device_count(C.byref(n)))
    return int(n.value)


class DeviceBuffer:
    """A device allocation with a numpy dtype/shape (bf16 is carried as uint16 bits)."""

    def __init__(self, ctx: Context, shape, dtype):
        self.ctx = ctx
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape)) * self.dtype.itemsize
        p = C.c_void_p()
        check(lib().k3cuda_malloc(ctx.h, C.byref(p), self.nbytes))
        self.ptr = p.value

    def free(self):
        if self.ptr:
            check(lib().k3cuda_free(self.ctx.h, self.ptr))
            self.ptr = None

    def __del__(self):
        try:
            if self.ptr and self.ctx.h:
                lib().k3cuda_free(self.ctx.h, self.ptr)
        except Exception:
            pass

    def copy_from(self, arr: np.ndarray):
        arr = np.ascontiguousarray(arr)
        assert arr.nbytes == self.nbytes, (arr.nbytes, self.nbytes)
        check(lib().k3cuda_memcpy_h2d(self.ctx.h, self.ptr, arr.ctypes.data, self.nbytes))
        self.ctx.sync()

    def copy_to(self, arr: np.ndarray):
        assert arr.nbytes == self.nbytes and arr.flags["C_CONTIGUOUS"]
        check(lib().k3cuda_memcpy_d2h(self.ctx.h, arr.ctypes.data, self.ptr, self.nbytes))
        self.ctx.sync()

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, self.dtype)
        self.copy_to(out)
        return out

    def zero(self):
        check(lib().k3cuda_memset(self.ctx.h, self.ptr, 0, self.nbytes))

    def fill(self, byte: int):
        """Set every byte to `byte` (asynchronous, on the context's stream)."""
        check(lib().k3cuda_memset(self.ctx.h, self.ptr, int(byte), self.nbytes))
