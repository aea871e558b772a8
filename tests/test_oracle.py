"""The CPU oracle pinned against the reference's golden vectors (CPU only).

Every check here compares oracle/k3_oracle.c (our restatement) either with the
reference's own fixtures (tests/fixtures/ops/*.json of the reference, converted by
tests/golden/make_golden.py) at the reference's MANIFEST tolerance, or with the reference C
compiled unmodified (oracle/_ref/libk3ref.so), bit for bit where both run the same fp32
arithmetic.
"""
import numpy as np
import pytest

from oracle import oracle
import workloads as W


def tol(golden):
    t = golden("manifest_tolerance")
    return float(t["fp32_abs"]), float(t["fp32_rel"])


def close(got, want, atol, rtol):
    """The reference harness's rule, |got - want| <= atol + rtol |want| (test_ops.c:114-131)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return bool(np.all(np.abs(got - want) <= atol + rtol * np.abs(want)))


@pytest.mark.parametrize("name", ["kda_recur1", "kda_recur8"])
def test_recurrence_matches_reference_fixture(golden, name):
    d = golden(name)
    T = d["q"].shape[0]
    o, S = oracle.kda_recurrence(d["q"], d["k"], d["v"], d["alpha"], d["beta"],
                                 np.array([0, T], np.int32), gate_is_log=False,
                                 q_scale=float(d["q_scale"]))
    atol, rtol = tol(golden)
    assert close(o, d["out"], atol, rtol)
    assert close(S[0], d["state_out"], atol, rtol)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("name", ["kda_recur1", "kda_recur8"])
def test_recurrence_bit_exact_with_reference_c(golden, name):
    d = golden(name)
    T = d["q"].shape[0]
    args = (d["q"], d["k"], d["v"], d["alpha"], d["beta"], np.array([0, T], np.int32))
    o1, S1 = oracle.kda_recurrence(*args, gate_is_log=False, q_scale=float(d["q_scale"]))
    o2, S2 = oracle.kda_recurrence(*args, gate_is_log=False, q_scale=float(d["q_scale"]),
                                   use_ref=True)
    assert np.array_equal(o1, o2) and np.array_equal(S1, S2)


def test_config0_golden_from_reference_c(golden):
    """BASELINE config 0 (T=256 prefill + 32 decode, H=4, d=64), reference C output."""
    d = golden("cfg0_kda")
    T = d["q"].shape[0]
    o, S = oracle.kda_recurrence(d["q"], d["k"], d["v"], d["g"], d["beta"],
                                 np.array([0, T], np.int32))
    assert np.array_equal(o, d["out"]) and np.array_equal(S, d["state_out"])


def test_config0_inputs_regenerate_from_seed(golden):
    d = golden("cfg0_kda")
    c0 = W.kda_config0()
    for key in ("q", "k", "v", "g", "beta"):
        assert np.array_equal(c0[key], d[key]), key


def test_decay_per_head(golden):
    d = golden("kda_decay")
    z = d["z"].reshape(-1, d["z"].shape[-1])
    H = d["A_log"].shape[0]
    D = z.shape[1] // H
    atol, rtol = tol(golden)
    for r in range(z.shape[0]):
        g = np.zeros(H * D, np.float32)
        a = np.zeros(H * D, np.float32)
        oracle.lib().orc_kda_decay(g, a, np.ascontiguousarray(z[r]), d["A_log"], d["dt_bias"], H,
                                   D, float(d["lower_bound"]))
        assert close(g, d["g"].reshape(z.shape[0], -1)[r], atol, rtol)
        assert close(a, d["alpha"].reshape(z.shape[0], -1)[r], atol, rtol)


@pytest.mark.parametrize("name", ["kda_layer1", "kda_layer8"])
def test_full_kda_layer_matches_reference_fixture(golden, name):
    d = golden(name)
    T, E = d["in"].shape[1], d["in"].shape[2]
    H, D, K = int(d["H"]), int(d["d_k"]), int(d["conv_k"])
    P = H * D
    state = np.zeros(H * D * D + 3 * P * (K - 1), np.float32)
    out = np.zeros((T, E), np.float32)
    f = lambda k: np.ascontiguousarray(d[k], np.float32)  # noqa: E731
    oracle.lib().orc_kda_layer(out, f("in"), T, E, H, D, K, float(d["lower_bound"]),
                               float(d["rms_eps"]), f("q_proj"), f("k_proj"), f("v_proj"),
                               f("q_conv"), f("k_conv"), f("v_conv"), f("f_a"), f("f_b"),
                               f("A_log"), f("dt_bias"), f("b_proj"), f("g_proj"), f("o_norm"),
                               f("o_proj"), state.ctypes.data)
    atol, rtol = tol(golden)
    assert close(out, d["out"][0], atol, rtol)
    assert close(state[: H * D * D], d["state_out"].ravel(), atol, rtol)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("wdt", [0, 1])
def test_kda_layer_bit_exact_with_reference_c(wdt):
    """orc_kda_layer against the reference's own k3_kda_layer (compiled from its sources) on
    a carried state: nonzero recurrent state and conv history, then calls of T = 1, 2 (both
    shorter than the conv history), 5 and 9 tokens, every output and the whole state
    bit-identical. wdt 1: bf16 projection weights (the real checkpoint's type) against the
    restatement run on the same weights widened to fp32."""
    rng = np.random.default_rng(40 + wdt)
    E, H, D, K = 256, 2, 128, 4
    w = W.kda_layer_weights(rng, E, H, D, K)
    if wdt:
        wr = {n: W.f32_to_bf16(w[n]) if n in oracle.LAYER_PROJ else w[n] for n in w}
        w = {n: W.bf16_to_f32(wr[n]) if n in oracle.LAYER_PROJ else w[n] for n in w}
    else:
        wr = w
    s_orc = (0.1 * rng.standard_normal(H * D * D + 3 * H * D * (K - 1))).astype(np.float32)
    s_ref = s_orc.copy()
    for T in (1, 2, 5, 9):
        x = rng.standard_normal((T, E)).astype(np.float32)
        a = oracle.kda_layer(x, w, H, D, K, -5.0, 1e-5, s_orc)
        b = oracle.ref_kda_layer(x, wr, H, D, K, -5.0, 1e-5, s_ref, wdt=wdt)
        assert np.array_equal(a, b), T
        assert np.array_equal(s_orc, s_ref), T


def test_absorbed_mla_matches_reference_expanded_cache(golden):
    """k3_mla_cached (expanded fp32 cache) vs the absorbed restatement, every causal prefix."""
    m = golden("mla_ref")
    P = m["q_nope"].shape[0]
    lat = np.broadcast_to(m["latent"], (P,) + m["latent"].shape[1:])
    rope = np.broadcast_to(m["rope"], (P,) + m["rope"].shape[1:])
    out = oracle.mla_absorbed_decode(m["q_nope"], m["q_rope"], lat, rope, m["w_uk"], m["w_uv"],
                                     m["ctx_lens"], float(m["scale"].item()))
    atol, rtol = tol(golden)
    assert close(out, m["out"], atol, rtol)
    assert W.rel_fro(out, m["out"]) < 1e-6


def test_chunked_restatement_matches_recurrence(golden):
    """The WY/UT chunk algebra (double) reproduces the token recurrence; its Akk/Aqk are
    the intra-chunk known answers the reference itself never forms."""
    d = golden("cfg0_kda")
    h = 1
    T = 256
    qs = 1.0 / np.sqrt(np.float32(64))
    oc, Sc, Akk, Aqk = oracle.kda_chunked_f64(d["q"][:T, h], d["k"][:T, h], d["v"][:T, h],
                                              d["g"][:T, h], d["beta"][:T, h], 64, qs)
    o1, S1 = oracle.kda_recurrence(d["q"][:T, h:h + 1], d["k"][:T, h:h + 1],
                                   d["v"][:T, h:h + 1], d["g"][:T, h:h + 1],
                                   d["beta"][:T, h:h + 1], np.array([0, T], np.int32))
    assert W.rel_fro(oc, o1[:, 0]) < 1e-5
    assert W.rel_fro(Sc, S1[0, 0]) < 1e-5
    # Akk strictly lower, Aqk lower with diagonal q.k
    assert np.all(np.triu(Akk[0]) == 0)
    assert np.allclose(np.diag(Aqk[0]),
                       np.sum(d["q"][:64, h].astype(np.float64) * qs * d["k"][:64, h], axis=1))


@pytest.mark.parametrize("d,decay", [(64, 1.0), (128, 1.0), (128, 6.0)])
def test_chunked_restatement_on_random_heads(d, decay):
    """The chunk algebra against the token recurrence on seeded random heads: both head widths
    the prefill kernels build, five chunks, and a decay strong enough (up to ~e^-6 per token)
    that the within-chunk factors span many orders of magnitude."""
    rng = np.random.default_rng(31 + d + int(decay))
    T = 5 * 64
    t = W.kda_tokens(rng, T, 1, d, d, bf16=False)
    g = (t["g"] * np.float32(decay)).astype(np.float32)
    qs = 1.0 / np.sqrt(np.float32(d))
    oc, Sc, _, _ = oracle.kda_chunked_f64(t["q"][:, 0], t["k"][:, 0], t["v"][:, 0], g[:, 0],
                                          t["beta"][:, 0], 64, qs)
    o1, S1 = oracle.kda_recurrence(t["q"], t["k"], t["v"], g, t["beta"],
                                   np.array([0, T], np.int32))
    assert W.rel_fro(oc, o1[:, 0]) < 1e-5
    assert W.rel_fro(Sc, S1[0, 0]) < 1e-5


def test_varlen_streams_are_independent():
    rng = np.random.default_rng(5)
    t = W.kda_tokens(rng, 50, 2, 16, 16, bf16=False)
    cu = np.array([0, 17, 17, 50], np.int32)
    o, S = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu)
    o2, S2 = oracle.kda_recurrence(t["q"][17:], t["k"][17:], t["v"][17:], t["g"][17:],
                                   t["beta"][17:], np.array([0, 33], np.int32))
    assert np.array_equal(o[17:], o2) and np.array_equal(S[2], S2[0])
    assert np.all(S[1] == 0)  # the empty sequence keeps its (zero) state


def test_bf16_round_trip():
    x = np.array([1.0, -2.5, 3.14159, 1e-30, 65504.0, 0.0], np.float32)
    b = W.f32_to_bf16(x)
    y = W.bf16_to_f32(b)
    assert np.array_equal(W.f32_to_bf16(y), b)
    assert np.all(np.abs(y - x) <= np.abs(x) * 2.0 ** -8)


def test_mxfp4_dequant_is_exact_on_checkpoint_bytes(golden):
    """orc_mxfp4_dequant on the reference's real checkpoint bytes (tests/fixtures/mxfp4.json):
    every value bit-exact (signed zeros too); the swapped nibble order gives the fixture's
    recorded wrong answer, so the order is really tested."""
    d = golden("mxfp4")
    got = oracle.mxfp4_dequant(d["packed"], d["scales"], int(d["group"]))
    assert np.array_equal(got.view(np.uint32), d["expected"].view(np.uint32))
    p = d["packed"]
    swapped = ((p & 15) << 4 | (p >> 4)).astype(np.uint8)
    wrong = oracle.mxfp4_dequant(swapped, d["scales"], int(d["group"]))
    assert np.array_equal(wrong[0, :64], d["expected_swapped_first64"])
    assert not np.array_equal(wrong, got)


def test_mxfp4_matmul_matches_reference(golden):
    """orc_matmul_mxfp4 against the reference's k3_matmul_mxfp4 output stored with the
    fixture (its own test bar: 1e-6 relative to dequantise-then-matmul)."""
    d = golden("mxfp4")
    y = oracle.matmul_mxfp4(d["x"], d["packed"], d["scales"], int(d["group"]))
    rel = np.abs(y - d["y_ref"]) / np.maximum(np.abs(d["y_ref"]), 1e-30)
    assert rel.max() < 1e-6


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("group,n_in", [(32, 256), (16, 96), (64, 130)])
def test_mxfp4_matmul_matches_reference_c_on_extreme_scales(group, n_in):
    """Random codes with scales at the extremes (0: subnormal 2^-127, 255: read as 0, up to
    2^100) and a partial last group, against the reference C directly."""
    rng = np.random.default_rng(group + n_in)
    rows = 37
    packed = rng.integers(0, 256, (rows, n_in // 2), dtype=np.uint8)
    ngrp = (n_in + group - 1) // group
    scales = rng.choice(np.array([0, 1, 100, 120, 127, 130, 200, 227, 255], np.uint8),
                        (rows, ngrp)).astype(np.uint8)
    x = rng.standard_normal((3, n_in)).astype(np.float32)
    want = oracle.matmul_mxfp4(x, packed, scales, group, use_ref=True)
    got = oracle.matmul_mxfp4(x, packed, scales, group)
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-30)
    assert rel.max() < 1e-6
    deq = oracle.mxfp4_dequant(packed, scales, group)
    ref = np.zeros_like(deq)
    oracle.ref().k3_mxfp4_dequant(ref, packed, scales, rows, n_in // 2, group)
    assert np.array_equal(deq.view(np.uint32), ref.view(np.uint32))
