"""Seeded synthetic inputs for the five workload configurations of the attention hot path.

The reference publishes no dataset for this path; every input is drawn from one seeded
numpy generator (PCG64) with the shapes and distributions below, and the SAME host arrays
feed the CUDA path and the CPU oracle:

  q, k   ~ N(0,1), L2-normalised per head per token (sum of squares + 1e-6 inside the
           square root, as the reference's l2norm_, src/core/k3_ops.c:845-851)
  v      ~ N(0,1)
  g      = -softplus(N(0,1)) per key channel, alpha = exp(g)
  beta   = sigmoid(N(0,1)) per head
  state  ~ N(0, 0.02^2) (0.02 read as the standard deviation)
  MLA:   q_nope, q_rope, rope cache ~ N(0,1); latent cache ~ N(0, 0.5^2) (0.5 read as the
         standard deviation); W_UK, W_UV ~ N(0, 0.02^2); scale 1/sqrt(128+64)

bf16 tensors are produced by rounding the fp32 draw to nearest-even and are carried as
uint16 bit patterns on the host; ``bf16_to_f32`` widens them exactly for the oracle.
"""
from __future__ import annotations

import numpy as np


# --------------------------------------------------------------------------- bf16
def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest-even), returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns to fp32 exactly (a 16-bit left shift, k3.h k3_bf16f)."""
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(x))


# --------------------------------------------------------------------------- draws
def _l2n(x: np.ndarray) -> np.ndarray:
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    return (x * (1.0 / np.sqrt(ss + 1e-6)).astype(np.float32)).astype(np.float32)


def _softplus(x: np.ndarray) -> np.ndarray:
    return np.logaddexp(np.float32(0), x).astype(np.float32)


def _sigmoid(x: np.ndarray) -> np.ndarray:
    return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


def kda_tokens(rng, T: int, H: int, dk: int, dv: int, bf16: bool):
    """q,k,v [T,H,d], g [T,H,dk] fp32, beta [T,H] fp32. With bf16=True q,k,v are rounded
    to bf16 (returned as fp32 values that are exactly representable in bf16)."""
    q = _l2n(rng.standard_normal((T, H, dk), dtype=np.float32))
    k = _l2n(rng.standard_normal((T, H, dk), dtype=np.float32))
    v = rng.standard_normal((T, H, dv), dtype=np.float32)
    g = -_softplus(rng.standard_normal((T, H, dk), dtype=np.float32))
    beta = _sigmoid(rng.standard_normal((T, H), dtype=np.float32))
    if bf16:
        q, k, v = round_bf16(q), round_bf16(k), round_bf16(v)
    return dict(q=q, k=k, v=v, g=g, beta=beta)


def kda_config0(seed: int = 0):
    """Config 0: B=1, prefill T=256 then 32 decode steps, H=4, d_k=d_v=64, fp32."""
    rng = np.random.default_rng(seed)
    return kda_tokens(rng, 256 + 32, 4, 64, 64, bf16=False)


def kda_config1(seed: int = 0, B: int = 256, H: int = 32, d: int = 128):
    """Config 1: one decode token for B sequences; fp32 state ~ N(0, 0.02^2)."""
    rng = np.random.default_rng(seed)
    t = kda_tokens(rng, B, H, d, d, bf16=True)
    S = (rng.standard_normal((B, H, d, d), dtype=np.float32) * np.float32(0.02))
    t["state"] = S
    return t


def kda_tokens_by_head(seed: int, T: int, H: int, dk: int, dv: int, bf16: bool,
                       heads: slice | None = None):
    """kda_tokens with one generator per head (seeded [seed, h]), so that any slice of
    heads -- a rank's head shard -- is drawn on its own and equals the same columns of the
    whole draw. Returns q, k, v [T, Hs, d], g [T, Hs, dk], beta [T, Hs]."""
    hs = range(H)[heads] if heads is not None else range(H)
    parts = [kda_tokens(np.random.default_rng([seed, h]), T, 1, dk, dv, bf16) for h in hs]
    return {x: np.ascontiguousarray(np.concatenate([p[x] for p in parts], axis=1))
            for x in ("q", "k", "v", "g", "beta")}


def kda_config2(seed: int = 0, T: int = 32768, H: int = 32, d: int = 128,
                heads: slice | None = None):
    """Config 2: one long sequence, bf16 q,k,v (`heads`: only that slice of the heads)."""
    t = kda_tokens_by_head(seed, T, H, d, d, True, heads)
    t["cu_seqlens"] = np.array([0, T], np.int32)
    return t


def varlen_lengths(seed: int = 0, nseq: int = 16, lo: int = 512, hi: int = 8192):
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=nseq).astype(np.int64)


def config3_cu_seqlens(seed: int = 0, nseq: int = 16, lo: int = 512, hi: int = 8192):
    lens = varlen_lengths(seed, nseq, lo, hi)
    cu = np.zeros(nseq + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    return cu


def kda_config3(seed: int = 0, nseq: int = 16, H: int = 64, d: int = 128, lo: int = 512,
                hi: int = 8192, heads: slice | None = None):
    """Config 3: packed variable-length batch, lengths ~ U[lo, hi] (seeded); `heads`: only
    that slice of the heads."""
    cu = config3_cu_seqlens(seed, nseq, lo, hi)
    t = kda_tokens_by_head(seed + 1, int(cu[-1]), H, d, d, True, heads)
    t["cu_seqlens"] = cu
    return t


def mla_config4(seed: int = 0, B: int = 64, ctx: int = 8192, H: int = 128, dn: int = 128,
                dr: int = 64, dl: int = 512, dv: int = 128):
    """Config 4: absorbed MLA decode inputs, every tensor bf16 (uint16 bits)."""
    rng = np.random.default_rng(seed)
    out = dict(
        q_nope=f32_to_bf16(rng.standard_normal((B, H, dn), dtype=np.float32)),
        q_rope=f32_to_bf16(rng.standard_normal((B, H, dr), dtype=np.float32)),
        latent=f32_to_bf16(rng.standard_normal((B, ctx, dl), dtype=np.float32) * np.float32(0.5)),
        rope=f32_to_bf16(rng.standard_normal((B, ctx, dr), dtype=np.float32)),
        w_uk=f32_to_bf16(rng.standard_normal((H, dn, dl), dtype=np.float32) * np.float32(0.02)),
        w_uv=f32_to_bf16(rng.standard_normal((H, dv, dl), dtype=np.float32) * np.float32(0.02)),
    )
    out["ctx_lens"] = np.full(B, ctx, np.int32)
    out["scale"] = float(1.0 / np.sqrt(np.float32(dn + dr)))
    return out


# KDA layer weight names as the reference's layer fixtures store them, in K3KdaW's field
# order (include/k3/k3.h:449-463), and the projections among them (the wdt-tagged ones).
LAYER_WEIGHTS = ("q_proj", "k_proj", "v_proj", "q_conv", "k_conv", "v_conv", "f_a", "f_b",
                 "A_log", "dt_bias", "b_proj", "g_proj", "o_norm", "o_proj")
LAYER_PROJ = ("q_proj", "k_proj", "v_proj", "f_a", "f_b", "b_proj", "g_proj", "o_proj")


def kda_layer_weights(rng, E: int, H: int, D: int, K: int = 4, pool: int = 0,
                      bf16: bool = False) -> dict:
    """Random weights of one KDA layer under the reference fixtures' names and shapes
    (tests/golden/kda_layer*.npz): entries N(0, 0.3) at fan-in 128, scaled by
    sqrt(128 / fan-in) so activations keep the fixtures' magnitude at any width; A_log in
    [-0.4, 1.2], dt_bias N(0.1, 0.45), o_norm 1 + N(0, 0.1). bf16: the projections are
    returned as bf16 bit patterns. pool > 0: each projection repeats one draw of `pool`
    values (model-size weights in seconds, for timing runs)."""
    P = H * D
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731

    def proj(rows, fan):
        n = rows * fan
        a = f(min(pool, n) if pool else n) * np.float32(0.3 * np.sqrt(128.0 / fan))
        if bf16:
            a = f32_to_bf16(a)
        return np.resize(a, (rows, fan)) if pool else a.reshape(rows, fan)

    return {
        "q_proj": proj(P, E), "k_proj": proj(P, E), "v_proj": proj(P, E),
        "g_proj": proj(P, E), "o_proj": proj(E, P), "f_a": proj(D, E),
        "f_b": proj(P, D), "b_proj": proj(H, E),
        "q_conv": f(P, 1, K) * np.float32(0.3), "k_conv": f(P, 1, K) * np.float32(0.3),
        "v_conv": f(P, 1, K) * np.float32(0.3),
        "A_log": rng.uniform(-0.4, 1.2, H).astype(np.float32),
        "dt_bias": (0.1 + 0.45 * f(P)).astype(np.float32),
        "o_norm": (1.0 + 0.1 * f(D)).astype(np.float32),
    }


def rel_fro(a: np.ndarray, b: np.ndarray) -> float:
    """Relative Frobenius error ||a - b||_F / ||b||_F in double."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))
