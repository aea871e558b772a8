"""The C ABI: both libraries load and export every function include/*.h declares (CPU only).

No kernel is launched here. The host-only parts of the ABI (argument checks, workspace
queries, error reporting) are exercised without a GPU.
"""
import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

import k3cuda
import workloads as W

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECL = re.compile(r"^\s*(?:const\s+)?(?:int|void|char|long\s+long|size_t)\s*\**\s*"
                  r"(k3cuda_\w+|k3g_\w+)\s*\(", re.M)


def declared(header):
    with open(os.path.join(ROOT, "include", header)) as f:
        return sorted(set(DECL.findall(f.read())))


def test_headers_declare_the_expected_entry_points():
    names = declared("k3cuda.h")
    for must in ("k3cuda_init", "k3cuda_kda_decode", "k3cuda_kda_prefill", "k3cuda_mla_decode",
                 "k3cuda_allgather_heads", "k3cuda_last_error"):
        assert must in names
    assert set(declared("k3_gpu.h")) >= {"k3g_kda_step", "k3g_kda_recurrence", "k3g_mla_attend"}


def test_every_header_symbol_is_exported_and_bound():
    L = k3cuda.lib()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        for name in declared(os.path.basename(h)):
            lib = k3cuda.gpu_lib() if name.startswith("k3g_") else L
            assert hasattr(lib, name), f"{name} declared in {h} but not exported"
            table = k3cuda.GPU_SIGNATURES if name.startswith("k3g_") else k3cuda.SIGNATURES
            assert name in table, f"{name} has no ctypes signature"


def test_library_is_sm100a_only():
    with open(os.path.join(ROOT, "kimi-k3-in-c_b200", "Makefile")) as f:
        mk = f.read()
    assert "arch=compute_100a,code=sm_100a" in mk


def test_workspace_queries_are_host_only():
    L = k3cuda.lib()
    cu = np.array([0, 100, 100, 300], np.int32)
    n = C.c_size_t()
    k3cuda.check(L.k3cuda_kda_prefill_workspace(cu.ctypes.data_as(C.POINTER(C.c_int)), 3, 4, 128,
                                                128, 64, C.byref(n)))
    nchunks = 2 + 0 + 4
    per_block = (3 * 64 * 128 + 128 + 2 * 64 * 64) * 4
    assert n.value >= nchunks * 4 * per_block
    # unsupported shapes and bad arguments are refused with a message, not a crash
    rc = L.k3cuda_kda_prefill_workspace(cu.ctypes.data_as(C.POINTER(C.c_int)), 3, 4, 96, 96, 64,
                                        C.byref(n))
    assert rc == k3cuda.ERR_UNSUPPORTED
    assert b"dk=96" in L.k3cuda_last_error()
    bad = np.array([0, 10, 5], np.int32)
    rc = L.k3cuda_kda_prefill_workspace(bad.ctypes.data_as(C.POINTER(C.c_int)), 2, 4, 128, 128,
                                        64, C.byref(n))
    assert rc == k3cuda.ERR_ARG
    cl = np.array([8192, 100], np.int32)
    k3cuda.check(L.k3cuda_mla_decode_workspace(cl.ctypes.data_as(C.POINTER(C.c_int)), 2, 128, 512,
                                               128, C.byref(n)))
    assert n.value > 2 * 128 * 576 * 4
    k3cuda.check(L.k3cuda_allgather_heads_workspace(8, 1000, 8, 128, k3cuda.BF16, C.byref(n)))
    assert n.value == 8 * 1000 * 8 * 128 * 2


def test_host_decode_staging_query():
    """The staging image of k3cuda_kda_decode_host: q, k, v, o in the io dtype, gate and beta in
    fp32, each region rounded up to 256 bytes; bad arguments are refused, not crashed on."""
    L = k3cuda.lib()
    n = C.c_size_t()
    ns = 256 * 32
    k3cuda.check(L.k3cuda_kda_decode_host_workspace(256, 32, 128, 128, k3cuda.BF16, C.byref(n)))
    assert n.value == 4 * ns * 128 * 2 + ns * 128 * 4 + ns * 4
    k3cuda.check(L.k3cuda_kda_decode_host_workspace(256, 32, 128, 128, k3cuda.F32, C.byref(n)))
    assert n.value == 5 * ns * 128 * 4 + ns * 4
    k3cuda.check(L.k3cuda_kda_decode_host_workspace(3, 1, 16, 16, k3cuda.BF16, C.byref(n)))
    assert n.value == 6 * 256  # every region of 3 x 16 values rounds up to 256 bytes
    assert L.k3cuda_kda_decode_host_workspace(3, 1, 16, 16, 7, C.byref(n)) == k3cuda.ERR_ARG
    assert L.k3cuda_kda_decode_host_workspace(-1, 1, 16, 16, k3cuda.BF16, C.byref(n)) == \
        k3cuda.ERR_ARG
    assert L.k3cuda_kda_decode_host_workspace(3, 1, 16, 16, k3cuda.BF16, None) == k3cuda.ERR_ARG


def test_init_without_gpu_fails_loudly():
    L = k3cuda.lib()
    cnt = C.c_int(0)
    rc = L.k3cuda_device_count(C.byref(cnt))
    if rc == 0 and cnt.value > 0:
        pytest.skip("a GPU is visible; the no-GPU error path is not reachable here")
    with pytest.raises(k3cuda.K3CudaError):
        k3cuda.Context(0)


def test_null_context_is_an_error_not_a_crash():
    L = k3cuda.lib()
    rc = L.k3cuda_kda_decode(None, None, None, None, None, None, None, None, 1, 1, 128, 128, 1.0,
                             k3cuda.BF16, k3cuda.GATE_LOG)
    assert rc == k3cuda.ERR_ARG
    assert L.k3cuda_last_error() == b"null context"


def test_workload_shapes():
    c = W.kda_config3(nseq=4, H=2, d=16, lo=10, hi=40)
    cu = c["cu_seqlens"]
    assert cu[0] == 0 and np.all(np.diff(cu) >= 10) and np.all(np.diff(cu) <= 40)
    assert c["q"].shape == (cu[-1], 2, 16)
    n = np.linalg.norm(c["q"].astype(np.float64), axis=-1)
    assert np.all(np.abs(n - 1) < 1e-2)
    assert np.all(c["g"] <= 0) and np.all((c["beta"] > 0) & (c["beta"] < 1))


def test_bench_unit_counts():
    """The algorithmic bytes and FLOPs that bench.py divides by (the roofline numerators) for the
    headline configurations, written out: each tensor a step must read or write once."""
    import importlib.util
    import os
    spec = importlib.util.spec_from_file_location(
        "bench_mod", os.path.join(os.path.dirname(__file__), "..", "bench.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    # config 1: fp32 state read + written, bf16 q, k, v, o, fp32 g and beta
    assert b.decode_bytes(256, 32, 128) == 1_086_357_504
    # config 2: 1540 B per (token, head) with bf16 q, k, v, o; 2564 B with fp32 ones
    assert b.prefill_bytes(32768, 32, 128) == 1_614_807_040 == 32768 * 32 * 1540
    assert b.prefill_bytes(32768, 32, 128, 4) == 2_688_548_864 == 32768 * 32 * 2564
    assert b.mla_bytes(64, 8192, 128) == 642_777_088
    assert b.layer_bytes(1, 7168, 96, 128, 4) == 900_685_824
    assert b.layer_flops(4096, 7168, 96, 128) == 2 * 4096 * (4 * 12288 * 7168 + 96 * 7168 +
                                                              128 * 7168 + 128 * 12288 +
                                                              12288 * 7168)
    assert b.mla_layer_bytes(1, 8192) == 473_882_624
    assert b.moe_expert_bytes() == 281_608_192
    assert b.mla_prefill_flops(4096, 128) == 2_474_471_587_840


def _mla_plan(lens, max_clusters=74):
    """(segments, clusters, exact workspace at H = 128) of the MLA attention work plan."""
    L = k3cuda.lib()
    arr = np.ascontiguousarray(lens, np.int32)
    ns, nc, nb = C.c_int(), C.c_int(), C.c_size_t()
    k3cuda.check(L.k3cuda_mla_plan_stats(arr.ctypes.data_as(C.POINTER(C.c_int)), len(arr),
                                         int(max_clusters), C.byref(ns), C.byref(nc),
                                         C.byref(nb)))
    return ns.value, nc.value, nb.value


def _mla_ws_query(lens, H=128):
    L = k3cuda.lib()
    arr = np.ascontiguousarray(lens, np.int32)
    n = C.c_size_t()
    k3cuda.check(L.k3cuda_mla_decode_workspace(arr.ctypes.data_as(C.POINTER(C.c_int)), len(arr),
                                               H, 512, 128, C.byref(n)))
    return n.value


def test_mla_work_plan_segments():
    """The attention work plan cuts the (query, tile) list into one contiguous run per cluster:
    every query gets at least one segment and a cluster boundary splits at most one query, so
    B <= segments <= B + clusters - 1 -- for a causal prefill (4096 queries of 1..4096
    positions, where the plan weighs each segment as extra tiles), for config 4 and for one
    long query (spread over 32 clusters by equal tile counts), on a full B200 and on parts
    with fewer SMs. The workspace query covers the plan of every cluster count."""
    for lens in (np.arange(1, 4097), np.full(64, 8192), np.array([8192]), np.array([1, 70, 3])):
        q = _mla_ws_query(lens)
        for mc in (74, 66, 37, 8, 1):
            nseg, ncl, need = _mla_plan(lens, mc)
            assert ncl <= mc
            assert len(lens) <= nseg <= len(lens) + ncl - 1, (len(lens), nseg, ncl, mc)
            assert need <= q, (len(lens), mc, need, q)
    nseg, ncl, _ = _mla_plan(np.array([8192]))
    assert ncl == 32 and nseg == 32


def test_dropin_structs_match_the_reference_layout(tmp_path):
    """k3g_cfg / k3g_kda_weights / k3g_mla_weights are K3Cfg / K3KdaW / K3MlaW field for field
    (the drop-ins are called through a cast): compile-time checks against the reference's own
    header, when a reference checkout is available to compile against."""
    import shutil
    import subprocess
    ref = os.environ.get("K3_REFERENCE_DIR", "")
    rec = os.path.join(ROOT, "oracle", "_ref", "refdir.txt")  # where the oracle was built from
    if not ref and os.path.exists(rec):
        with open(rec) as f:
            ref = f.read().strip()
    hdr = os.path.join(ref, "include", "k3", "k3.h")
    if not os.path.isfile(hdr) or not shutil.which("gcc"):
        pytest.skip("no reference checkout to compile against")
    src = tmp_path / "layout.c"
    fields = {"K3Cfg": ("k3g_cfg", ["hidden", "n_layers", "vocab", "rms_eps", "kda_heads",
                                    "kda_head_dim", "conv_k", "gate_lb", "n_heads", "q_lora",
                                    "kv_lora", "qk_nope", "qk_rope", "v_head", "mla_out_gate",
                                    "n_experts", "topk", "n_shared", "latent", "moe_inter",
                                    "routed_scale", "moe_renorm", "latent_norm", "first_dense",
                                    "dense_inter", "attn_res_block", "situ_b1", "situ_b2",
                                    "n_full_attn", "full_attn"]),
              "K3KdaW": ("k3g_kda_weights", ["q", "k", "v", "q_conv", "k_conv", "v_conv", "f_a",
                                             "f_b", "A_log", "dt_bias", "b", "g", "o_norm", "o",
                                             "wdt"]),
              "K3MlaW": ("k3g_mla_weights", ["q_a", "q_b", "kv_a", "kv_b", "o", "g", "q_a_norm",
                                             "kv_a_norm", "wdt"])}
    lines = ["#include <stddef.h>", '#include "k3.h"', '#include "k3_gpu.h"']
    for ref_t, (our_t, names) in fields.items():
        lines.append(f'_Static_assert(sizeof({ref_t}) == sizeof({our_t}), "{ref_t} size");')
        for n in names:
            lines.append(f"_Static_assert(offsetof({ref_t}, {n}) == offsetof({our_t}, {n}) && "
                         f"sizeof((({ref_t} *)0)->{n}) == sizeof((({our_t} *)0)->{n}), "
                         f'"{ref_t}.{n}");')
    src.write_text("\n".join(lines) + "\n")
    inc = [f"-I{ref}/include", f"-I{ref}/include/k3", f"-I{ref}/third_party",
           f"-I{os.path.join(ROOT, 'include')}"]
    r = subprocess.run(["gcc", "-std=gnu99", "-fsyntax-only", *inc, str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
