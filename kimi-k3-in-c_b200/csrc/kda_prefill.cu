// kda_prefill.cu -- KDA chunkwise prefill over packed variable-length sequences.
//
// Replaces the token-by-token recurrence of k3_kda_layer (reference src/core/k3_ops.c:
// 908-938, k3_kda_step at :186-243) with the chunkwise (WY / UT-transform) form of the
// gated delta rule. Inside a chunk of C = 64 tokens with per-channel cumulative log decay
// G_t = sum_{u<=t} g_u:
//     (I + Akk) Delta = diag(beta) (V - Ktil S0)     Akk[t][s] = beta_t sum_i k_ti k_si e^(G_ti - G_si), s < t
//     O   = Qtil S0 + Aqk Delta                      Aqk[t][s] = sum_i q_ti k_si e^(G_ti - G_si),      s <= t
//     S_C = diag(e^G_C) S0 + Kbar^T Delta
// with Ktil_t = e^G_t k_t, Qtil_t = e^G_t q_t (q pre-multiplied by q_scale) and
// Kbar_s = e^(G_C - G_s) k_s. Every factor above is <= 1, so nothing overflows.
//
// Two kernels:
//   kda_chunk_intra  one CTA per (chunk, head), all chunks in parallel: G, Akk, Aqk with
//                    16-token sub-block anchors, M = (I + Akk)^-1 diag(beta) by forward
//                    substitution, and the scaled operands Qtil, Ktil, Kbar, e^G_C.
//   kda_chunk_scan   one CTA per (sequence, head, 16-column slice of d_v): walks the
//                    sequence's chunks in order with its state slice in shared memory:
//                    X = V - Ktil S; Delta = M X; O = Qtil S + Aqk Delta;
//                    S = e^G_C S + Kbar^T Delta.
// Columns of the state are independent in every step, which is what lets the scan split
// d_v across CTAs with no communication.
//
// Anchors. e^(G_t - G_s) is formed as e^(G_t - G_r) e^(G_r - G_s) with r the first token
// of t's 16-token sub-block. For s before the sub-block both factors are <= 1. For s
// inside it e^(G_r - G_s) >= 1 spans at most 15 decay steps; if any channel's 15-step
// decay exceeds e^80 the sub-block's diagonal entries are formed directly instead.
#include <type_traits>
#include <vector>

#include <string.h>

#include <algorithm>

#include "internal.cuh"

namespace k3 {

// kda_prefill_tc.cu: the tcgen05 form, used for bf16 q/k/v/o with d_k = d_v = 128
int run_prefill_tc(k3cuda_ctx *ctx, float *state, void *o, const void *q, const void *k,
                   const void *v, const float *gate, const float *beta, int total_tokens,
                   int n_seq, int H, float q_scale, int gate_is_log, long long nc,
                   const void *d_table, const int *d_c0, void *blocks, const GatherOut *go);
size_t prefill_tc_block_bytes();

constexpr int KC = 64;        // chunk length
constexpr int KSUB = 16;      // anchor sub-block
constexpr int SCAN_DVT = 16;  // d_v columns per scan CTA

struct ChunkDesc {
    int seq;    // sequence index
    int t0;     // first token (packed index)
    int len;    // tokens in this chunk (1..64)
    int pad;
};

template <int DK>
struct PrefillLayout {
    // per (chunk, head) block, in floats
    static constexpr size_t qt = 0;
    static constexpr size_t kt = qt + (size_t)KC * DK;
    static constexpr size_t kb = kt + (size_t)KC * DK;
    static constexpr size_t gc = kb + (size_t)KC * DK;
    static constexpr size_t m = gc + DK;
    static constexpr size_t aqk = m + (size_t)KC * KC;
    static constexpr size_t floats = aqk + (size_t)KC * KC;
};

__device__ __forceinline__ float load_gate(const float *p, int gate_is_log) {
    const float x = *p;
    return gate_is_log ? x : logf(x);
}

// ---------------------------------------------------------------------------- intra
template <typename IO, int DK>
__global__ void __launch_bounds__(256, 1)
kda_chunk_intra(const ChunkDesc *__restrict__ chunks, const IO *__restrict__ q,
                const IO *__restrict__ k, const float *__restrict__ gate,
                const float *__restrict__ beta, float *__restrict__ ws, int H, float q_scale,
                int gate_is_log) {
    using L = PrefillLayout<DK>;
    extern __shared__ __align__(16) float sm[];
    float *sk = sm;                     // [KC][DK]  k
    float *sq = sk + KC * DK;           // [KC][DK]  q * q_scale
    float *sG = sq + KC * DK;           // [KC][DK]  cumulative log decay
    float *sKh = sG + KC * DK;          // [KC][DK]  k_s e^(G_r - G_s) for the current anchor r
    float *sKa = sKh + KC * DK;         // [KSUB][DK] k_t e^(G_t - G_r)
    float *sQa = sKa + KSUB * DK;       // [KSUB][DK] q_t e^(G_t - G_r)
    float *sA = sQa + KSUB * DK;        // [KC][KC]  Akk (beta-scaled, strictly lower)
    float *sAq = sA + KC * KC;          // [KC][KC]  Aqk (lower incl. diagonal)
    float *sT = sAq + KC * KC;          // [KC][KC]  (I + Akk)^-1
    float *sb = sT + KC * KC;           // [KC]      beta

    const ChunkDesc cd = chunks[blockIdx.x];
    const int h = blockIdx.y, tid = threadIdx.x;
    float *out = ws + ((size_t)blockIdx.x * H + h) * L::floats;

    for (int e = tid; e < KC * DK; e += 256) {
        const int t = e / DK, i = e - t * DK;
        float kv = 0.f, qv = 0.f, gv = 0.f;
        if (t < cd.len) {
            const size_t off = ((size_t)(cd.t0 + t) * H + h) * DK + i;
            kv = io<IO>::ld(k + off);
            qv = io<IO>::ld(q + off) * q_scale;
            gv = load_gate(gate + off, gate_is_log);
        }
        sk[e] = kv;
        sq[e] = qv;
        sG[e] = gv;
    }
    if (tid < KC) sb[tid] = tid < cd.len ? beta[(size_t)(cd.t0 + tid) * H + h] : 0.f;
    __syncthreads();
    if (tid < DK) {
        float acc = 0.f;
        for (int t = 0; t < KC; t++) {
            acc += sG[t * DK + tid];
            sG[t * DK + tid] = acc;
        }
    }
    __syncthreads();

    // scaled operands for the scan (full-chunk anchor at the chunk start)
    for (int e = tid; e < KC * DK; e += 256) {
        const int t = e / DK, i = e - t * DK;
        const float G = sG[e], GC = sG[(KC - 1) * DK + i];
        const float eg = expf(G);
        out[L::qt + e] = sq[e] * eg;
        out[L::kt + e] = sk[e] * eg;
        out[L::kb + e] = sk[e] * expf(GC - G);
    }
    if (tid < DK) out[L::gc + tid] = expf(sG[(KC - 1) * DK + tid]);

    // Akk / Aqk, one 16-row sub-block at a time
    for (int a = 0; a < KC / KSUB; a++) {
        const int r0 = a * KSUB, ncol = r0 + KSUB;
        int big = 0;
        for (int e = tid; e < ncol * DK; e += 256) {
            const int s = e / DK, i = e - s * DK;
            const float ex = sG[r0 * DK + i] - sG[e];
            big |= ex > 80.f;
            sKh[e] = sk[e] * expf(fminf(ex, 80.f));
        }
        for (int e = tid; e < KSUB * DK; e += 256) {
            const int t = r0 + e / DK, i = e % DK;
            const float f = expf(sG[t * DK + i] - sG[r0 * DK + i]);
            sKa[e] = sk[t * DK + i] * f;
            sQa[e] = sq[t * DK + i] * f;
        }
        big = __syncthreads_or(big);
        for (int e = tid; e < KSUB * KC; e += 256) {
            const int tl = e / KC, s = e - tl * KC, t = r0 + tl;
            float akk = 0.f, aqk = 0.f;
            if (s <= t) {
                if (big && s >= r0) {
                    for (int i = 0; i < DK; i++) {
                        const float f = expf(sG[t * DK + i] - sG[s * DK + i]) * sk[s * DK + i];
                        akk += sk[t * DK + i] * f;
                        aqk += sq[t * DK + i] * f;
                    }
                } else {
                    const float *ka = sKa + tl * DK, *qa = sQa + tl * DK, *kh = sKh + s * DK;
                    for (int i = 0; i < DK; i++) {
                        akk += ka[i] * kh[i];
                        aqk += qa[i] * kh[i];
                    }
                }
            }
            sA[t * KC + s] = s < t ? sb[t] * akk : 0.f;
            sAq[t * KC + s] = aqk;
        }
        __syncthreads();
    }

    // T = (I + Akk)^-1 by forward substitution, row by row; M = T diag(beta)
    for (int e = tid; e < KC * KC; e += 256) sT[e] = (e / KC == e % KC) ? 1.f : 0.f;
    __syncthreads();
    for (int t = 1; t < KC; t++) {
        if (tid < t) {
            const int s = tid;
            float acc = 0.f;
            for (int j = s; j < t; j++) acc += sA[t * KC + j] * sT[j * KC + s];
            sT[t * KC + s] = -acc;
        }
        __syncthreads();
    }
    for (int e = tid; e < KC * KC; e += 256) {
        const int s = e % KC;
        out[L::m + e] = sT[e] * sb[s];
        out[L::aqk + e] = sAq[e];
    }
}

// ----------------------------------------------------------------------------- scan
template <typename IO, int DK>
__global__ void __launch_bounds__(256, 1)
kda_chunk_scan(const ChunkDesc *__restrict__ chunks, const int *__restrict__ seq_chunk0,
               const IO *__restrict__ v, const float *__restrict__ ws, float *__restrict__ state,
               IO *__restrict__ o, int H) {
    using L = PrefillLayout<DK>;
    constexpr int DV = DK, NT = DV / SCAN_DVT;
    extern __shared__ __align__(16) float sm[];
    float *sQt = sm;                    // [KC][DK]
    float *sKt = sQt + KC * DK;         // [KC][DK]
    float *sKb = sKt + KC * DK;         // [KC][DK]
    float *sM = sKb + KC * DK;          // [KC][KC]
    float *sAq = sM + KC * KC;          // [KC][KC]
    float *sS = sAq + KC * KC;          // [DK][SCAN_DVT]
    float *sX = sS + DK * SCAN_DVT;     // [KC][SCAN_DVT]
    float *sD = sX + KC * SCAN_DVT;     // [KC][SCAN_DVT]
    float *sGc = sD + KC * SCAN_DVT;    // [DK]

    const int tile = blockIdx.x % NT;
    const int h = (blockIdx.x / NT) % H;
    const int n = blockIdx.x / (NT * H);
    const int tid = threadIdx.x, j = tid % SCAN_DVT, r = tid / SCAN_DVT;  // r in 0..15
    const int c0 = seq_chunk0[n], c1 = seq_chunk0[n + 1];
    const int col0 = tile * SCAN_DVT;
    float *Sg = state ? state + ((size_t)n * H + h) * DK * DV : nullptr;

    for (int e = tid; e < DK * SCAN_DVT; e += 256) {
        const int i = e / SCAN_DVT, jj = e % SCAN_DVT;
        sS[e] = Sg ? Sg[(size_t)i * DV + col0 + jj] : 0.f;
    }
    for (int c = c0; c < c1; c++) {
        const ChunkDesc cd = chunks[c];
        const float *blk = ws + ((size_t)c * H + h) * L::floats;
        __syncthreads();
        for (int e = tid; e < KC * DK / 4; e += 256) {
            reinterpret_cast<float4 *>(sQt)[e] = reinterpret_cast<const float4 *>(blk + L::qt)[e];
            reinterpret_cast<float4 *>(sKt)[e] = reinterpret_cast<const float4 *>(blk + L::kt)[e];
            reinterpret_cast<float4 *>(sKb)[e] = reinterpret_cast<const float4 *>(blk + L::kb)[e];
        }
        for (int e = tid; e < KC * KC / 4; e += 256) {
            reinterpret_cast<float4 *>(sM)[e] = reinterpret_cast<const float4 *>(blk + L::m)[e];
            reinterpret_cast<float4 *>(sAq)[e] = reinterpret_cast<const float4 *>(blk + L::aqk)[e];
        }
        if (tid < DK) sGc[tid] = blk[L::gc + tid];
        // X = V - Ktil S
        for (int t = r; t < KC; t += 16) {
            float vv = 0.f;
            if (t < cd.len) vv = io<IO>::ld(v + ((size_t)(cd.t0 + t) * H + h) * DV + col0 + j);
            sX[t * SCAN_DVT + j] = vv;
        }
        __syncthreads();
        for (int t = r; t < KC; t += 16) {
            float acc = 0.f;
            const float *kt = sKt + t * DK;
            for (int i = 0; i < DK; i++) acc += kt[i] * sS[i * SCAN_DVT + j];
            sX[t * SCAN_DVT + j] -= acc;
        }
        __syncthreads();
        // Delta = M X  (M lower triangular)
        for (int t = r; t < KC; t += 16) {
            float acc = 0.f;
            const float *m = sM + t * KC;
            for (int s = 0; s <= t; s++) acc += m[s] * sX[s * SCAN_DVT + j];
            sD[t * SCAN_DVT + j] = acc;
        }
        __syncthreads();
        // O = Qtil S + Aqk Delta
        for (int t = r; t < cd.len; t += 16) {
            float acc = 0.f;
            const float *qt = sQt + t * DK;
            for (int i = 0; i < DK; i++) acc += qt[i] * sS[i * SCAN_DVT + j];
            const float *aq = sAq + t * KC;
            for (int s = 0; s <= t; s++) acc += aq[s] * sD[s * SCAN_DVT + j];
            io<IO>::st(o + ((size_t)(cd.t0 + t) * H + h) * DV + col0 + j, acc);
        }
        __syncthreads();
        // S = e^G_C S + Kbar^T Delta
        for (int i = r; i < DK; i += 16) {
            float acc = sGc[i] * sS[i * SCAN_DVT + j];
            for (int s = 0; s < KC; s++) acc += sKb[s * DK + i] * sD[s * SCAN_DVT + j];
            sS[i * SCAN_DVT + j] = acc;
        }
    }
    __syncthreads();
    if (Sg)
        for (int e = tid; e < DK * SCAN_DVT; e += 256) {
            const int i = e / SCAN_DVT, jj = e % SCAN_DVT;
            Sg[(size_t)i * DV + col0 + jj] = sS[e];
        }
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static int count_chunks(const int *cu, int n_seq, long long *nc) {
    long long c = 0;
    for (int n = 0; n < n_seq; n++) {
        const int len = cu[n + 1] - cu[n];
        if (len < 0) return set_error(K3CUDA_ERR_ARG, "cu_seqlens not non-decreasing at %d", n);
        c += (len + KC - 1) / KC;
    }
    *nc = c;
    return K3CUDA_OK;
}

// chunk table, then the sequences' first-chunk offsets [n_seq + 1] and the sequences in
// descending chunk count [n_seq] (the order the tensor-core scan takes them: the longest
// chains start first and the short ones fill in behind them)
static size_t table_bytes(long long nc, int n_seq) {
    return align256((size_t)nc * sizeof(ChunkDesc)) +
           align256((size_t)(2 * n_seq + 1) * sizeof(int));
}

template <typename IO, int DK>
static int run_prefill(k3cuda_ctx *ctx, float *state, void *o, const void *q, const void *k,
                       const void *v, const float *gate, const float *beta, const int *cu,
                       int n_seq, int H, float q_scale, int gate_is_log, long long nc,
                       void *workspace, const GatherOut *go = nullptr) {
    using L = PrefillLayout<DK>;
    std::vector<ChunkDesc> table((size_t)nc);
    std::vector<int> c0((size_t)2 * n_seq + 1);
    long long c = 0;
    for (int n = 0; n < n_seq; n++) {
        c0[n] = (int)c;
        for (int t = cu[n]; t < cu[n + 1]; t += KC) {
            const int len = cu[n + 1] - t < KC ? cu[n + 1] - t : KC;
            table[(size_t)c++] = ChunkDesc{n, t, len, 0};
        }
    }
    c0[n_seq] = (int)c;
    {
        std::vector<int> ord((size_t)n_seq);
        for (int n = 0; n < n_seq; n++) ord[(size_t)n] = n;
        std::stable_sort(ord.begin(), ord.end(), [&](int a, int b) {
            return c0[(size_t)a + 1] - c0[(size_t)a] > c0[(size_t)b + 1] - c0[(size_t)b];
        });
        for (int n = 0; n < n_seq; n++) c0[(size_t)n_seq + 1 + n] = ord[(size_t)n];
    }
    char *wsb = (char *)workspace;
    ChunkDesc *d_table = (ChunkDesc *)wsb;
    int *d_c0 = (int *)(wsb + align256((size_t)nc * sizeof(ChunkDesc)));
    float *blocks = (float *)(wsb + table_bytes(nc, n_seq));
    {
        // the chunk table and the sequence offsets are adjacent: one image, one copy
        std::vector<unsigned char> img(table_bytes(nc, n_seq), 0);
        if (nc > 0) memcpy(img.data(), table.data(), (size_t)nc * sizeof(ChunkDesc));
        memcpy(img.data() + ((char *)d_c0 - wsb), c0.data(), c0.size() * sizeof(int));
        if (int rc = stage_h2d(ctx, wsb, img.data(), img.size())) return rc;
    }
    if constexpr (std::is_same<IO, __nv_bfloat16>::value && DK == 128) {
        // bf16 operands on the tensor cores (every operand bf16, accumulation fp32)
        if (nc == 0) return K3CUDA_OK;
        return run_prefill_tc(ctx, state, o, q, k, v, gate, beta, cu[n_seq], n_seq, H, q_scale,
                              gate_is_log, nc, d_table, d_c0, blocks, go);
    }
    if (nc > 0) {
        const size_t smem1 =
            ((size_t)4 * KC * DK + 2 * KSUB * DK + 3 * KC * KC + KC) * sizeof(float);
        if (int rc_ = set_smem(kda_chunk_intra<IO, DK>, (int)smem1)) return rc_;
        dim3 g1((unsigned)nc, (unsigned)H);
        kda_chunk_intra<IO, DK><<<g1, 256, smem1, ctx->stream>>>(
            d_table, (const IO *)q, (const IO *)k, gate, beta, blocks, H, q_scale, gate_is_log);
        int rc = after_launch(ctx, "kda_chunk_intra");
        if (rc) return rc;
    }
    const size_t smem2 = ((size_t)3 * KC * DK + 2 * KC * KC + DK * SCAN_DVT + 2 * KC * SCAN_DVT +
                          DK) * sizeof(float);
    if (int rc_ = set_smem(kda_chunk_scan<IO, DK>, (int)smem2)) return rc_;
    const long long nblk = (long long)n_seq * H * (DK / SCAN_DVT);
    if (nblk > 0) {
        kda_chunk_scan<IO, DK><<<(unsigned)nblk, 256, smem2, ctx->stream>>>(
            d_table, d_c0, (const IO *)v, blocks, state, (IO *)o, H);
        return after_launch(ctx, "kda_chunk_scan");
    }
    (void)L::floats;
    return K3CUDA_OK;
}

}  // namespace k3

using namespace k3;

extern "C" int k3cuda_kda_prefill_workspace(const int *cu_seqlens, int n_seq, int H, int dk,
                                            int dv, int chunk, size_t *bytes) {
    K3_ARG_CHECK(bytes && cu_seqlens && n_seq >= 0 && H >= 1, "bad prefill workspace query");
    if (chunk != KC || dk != dv || (dk != 64 && dk != 128))
        return set_error(K3CUDA_ERR_UNSUPPORTED, "kda_prefill: dk=%d dv=%d chunk=%d not built",
                         dk, dv, chunk);
    long long nc = 0;
    int rc = count_chunks(cu_seqlens, n_seq, &nc);
    if (rc) return rc;
    const size_t per = dk == 64 ? PrefillLayout<64>::floats : PrefillLayout<128>::floats;
    *bytes = table_bytes(nc, n_seq) + (size_t)nc * H * per * sizeof(float);
    return K3CUDA_OK;
}

extern "C" int k3cuda_kda_prefill(k3cuda_ctx *ctx, float *state, void *o, const void *q,
                                  const void *k, const void *v, const float *gate,
                                  const float *beta, const int *cu_seqlens, int n_seq, int H,
                                  int dk, int dv, float q_scale, int io_dtype, int gate_mode,
                                  int chunk, void *workspace, size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(io_dtype == K3CUDA_F32 || io_dtype == K3CUDA_BF16, "bad io_dtype %d", io_dtype);
    K3_ARG_CHECK(gate_mode == K3CUDA_GATE_LOG || gate_mode == K3CUDA_GATE_ALPHA,
                 "bad gate_mode %d", gate_mode);
    size_t need = 0;
    rc = k3cuda_kda_prefill_workspace(cu_seqlens, n_seq, H, dk, dv, chunk, &need);
    if (rc) return rc;
    if (cu_seqlens[0] != 0) return set_error(K3CUDA_ERR_ARG, "cu_seqlens[0] must be 0");
    if (workspace_bytes < need || (need && !workspace))
        return set_error(K3CUDA_ERR_WORKSPACE, "kda_prefill: workspace %zu < %zu bytes",
                         workspace_bytes, need);
    K3_ARG_CHECK(aligned(workspace, 256), "workspace must be 256-byte aligned");
    if (cu_seqlens[n_seq] == 0 || n_seq == 0) return K3CUDA_OK;
    K3_ARG_CHECK(o && q && k && v && gate && beta, "kda_prefill: null pointer");
    long long nc = 0;
    count_chunks(cu_seqlens, n_seq, &nc);
    const int gl = gate_mode == K3CUDA_GATE_LOG;
    if (io_dtype == K3CUDA_BF16) {
        if (dk == 64)
            return run_prefill<__nv_bfloat16, 64>(ctx, state, o, q, k, v, gate, beta, cu_seqlens,
                                                  n_seq, H, q_scale, gl, nc, workspace);
        return run_prefill<__nv_bfloat16, 128>(ctx, state, o, q, k, v, gate, beta, cu_seqlens,
                                               n_seq, H, q_scale, gl, nc, workspace);
    }
    if (dk == 64)
        return run_prefill<float, 64>(ctx, state, o, q, k, v, gate, beta, cu_seqlens, n_seq, H,
                                      q_scale, gl, nc, workspace);
    return run_prefill<float, 128>(ctx, state, o, q, k, v, gate, beta, cu_seqlens, n_seq, H,
                                   q_scale, gl, nc, workspace);
}

// ------------------------------------------------- head-sharded prefill, gathered output
namespace k3 {
// comm.cu: a one-int all-reduce ordering all ranks (wait_host: the host also waits for it,
// under the communicator's deadline)
int comm_fence(k3cuda_ctx *ctx, bool wait_host);
// comm.cu: copy this rank's heads of its full buffer into every peer's full buffer
int comm_push_heads(k3cuda_ctx *ctx, int T, int head0, int H_local, int H_total, int dv);
}

extern "C" int k3cuda_kda_prefill_gathered(k3cuda_ctx *ctx, float *state, const void *q,
                                           const void *k, const void *v, const float *gate,
                                           const float *beta, const int *cu_seqlens, int n_seq,
                                           int H_local, int dk, int dv, float q_scale,
                                           int gate_mode, int chunk, void *workspace,
                                           size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (ctx->comm_failed)
        return set_error(K3CUDA_ERR_STATE, "the communicator was aborted after a failure");
    if (!ctx->nccl_comm || !ctx->full_out[ctx->rank])
        return set_error(K3CUDA_ERR_STATE,
                         "kda_prefill_gathered: k3cuda_comm_init and k3cuda_comm_register_full "
                         "first");
    K3_ARG_CHECK(dk == 128 && dv == 128, "kda_prefill_gathered: built for dk = dv = 128 only");
    K3_ARG_CHECK(gate_mode == K3CUDA_GATE_LOG || gate_mode == K3CUDA_GATE_ALPHA,
                 "bad gate_mode %d", gate_mode);
    size_t need = 0;
    rc = k3cuda_kda_prefill_workspace(cu_seqlens, n_seq, H_local, dk, dv, chunk, &need);
    if (rc) return rc;
    if (cu_seqlens[0] != 0) return set_error(K3CUDA_ERR_ARG, "cu_seqlens[0] must be 0");
    if (workspace_bytes < need || (need && !workspace))
        return set_error(K3CUDA_ERR_WORKSPACE, "kda_prefill_gathered: workspace %zu < %zu bytes",
                         workspace_bytes, need);
    K3_ARG_CHECK(aligned(workspace, 256), "workspace must be 256-byte aligned");
    const int T = cu_seqlens[n_seq];
    const size_t full_need = (size_t)T * ctx->nranks * H_local * dv * 2;
    if (full_need > ctx->full_bytes)
        return set_error(K3CUDA_ERR_ARG,
                         "kda_prefill_gathered: output needs %zu bytes, registered buffer has %zu",
                         full_need, ctx->full_bytes);
    K3_ARG_CHECK(T == 0 || (q && k && v && gate && beta), "kda_prefill_gathered: null pointer");
    // the scan writes this rank's heads straight into its own full buffer (final layout);
    // one coalesced pass then pushes that head span into every peer's buffer over NVLink
    GatherOut go{};
    go.ptr[0] = (__nv_bfloat16 *)ctx->full_out[ctx->rank];
    go.n = 1;
    go.head0 = ctx->rank * H_local;
    go.H_total = ctx->nranks * H_local;
    // every rank is done with the previous contents of its buffer before anyone writes; the
    // host sees this fence complete before it enqueues any peer store, so a peer that has
    // gone (or stalled past the deadline) ends the call with an error, never with a store
    // into a buffer whose owner has left
    rc = comm_fence(ctx, true);
    if (rc) return rc;
    if (T > 0 && n_seq > 0) {
        long long nc = 0;
        count_chunks(cu_seqlens, n_seq, &nc);
        rc = run_prefill<__nv_bfloat16, 128>(ctx, state, nullptr, q, k, v, gate, beta,
                                             cu_seqlens, n_seq, H_local, q_scale,
                                             gate_mode == K3CUDA_GATE_LOG, nc, workspace, &go);
        if (rc) return rc;
        rc = comm_push_heads(ctx, T, go.head0, H_local, go.H_total, dv);
        if (rc) return rc;
    }
    // and every rank's writes into every buffer are complete before anyone reads one
    return comm_fence(ctx, false);
}

// ------------------------------------------------------------- allocation-free variant
// Some callers cannot allocate device memory at the point they run a prefill: a host
// runtime that has already reserved the whole HBM budget through its own allocator, or a
// latency-critical path where cudaMalloc's implicit device synchronisation would stall
// other streams. For them the workspace of k3cuda_kda_prefill lives in this file-scope
// array instead, K3CUDA_NOALLOC_SCRATCH_BYTES on every GPU that loads the library, held
// until the process exits.
#include <mutex>

static __device__ __align__(256) unsigned char g_prefill_scratch[K3CUDA_NOALLOC_SCRATCH_BYTES];

namespace k3 {
static std::mutex g_scratch_mu;
static void *g_scratch_dev[256];  // device address of g_prefill_scratch, per device ordinal
}  // namespace k3

extern "C" int k3cuda_kda_prefill_noalloc(k3cuda_ctx *ctx, float *state, void *o, const void *q,
                                          const void *k, const void *v, const float *gate,
                                          const float *beta, const int *cu_seqlens, int n_seq,
                                          int H, int dk, int dv, float q_scale, int io_dtype,
                                          int gate_mode, int chunk) {
    int rc = enter(ctx);
    if (rc) return rc;
    size_t need = 0;
    rc = k3cuda_kda_prefill_workspace(cu_seqlens, n_seq, H, dk, dv, chunk, &need);
    if (rc) return rc;
    if (need > K3CUDA_NOALLOC_SCRATCH_BYTES)
        return set_error(K3CUDA_ERR_WORKSPACE,
                         "kda_prefill_noalloc: this call needs %zu bytes of scratch; the static "
                         "scratch holds %zu (split the batch, or use k3cuda_kda_prefill)",
                         need, (size_t)K3CUDA_NOALLOC_SCRATCH_BYTES);
    if (ctx->device < 0 || ctx->device >= 256)
        return set_error(K3CUDA_ERR_ARG, "device ordinal %d out of range", ctx->device);
    void *scratch;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_dev[ctx->device]) {
            // set-up, once per device, with the device current (enter() made it so)
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_prefill_scratch);
            if (e != cudaSuccess || !p)
                return set_error(K3CUDA_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s",
                                 cudaGetErrorString(e));
            g_scratch_dev[ctx->device] = p;
        }
        scratch = g_scratch_dev[ctx->device];
    }
    return k3cuda_kda_prefill(ctx, state, o, q, k, v, gate, beta, cu_seqlens, n_seq, H, dk, dv,
                              q_scale, io_dtype, gate_mode, chunk, scratch,
                              K3CUDA_NOALLOC_SCRATCH_BYTES);
}
