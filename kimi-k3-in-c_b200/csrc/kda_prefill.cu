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
// Kernels (bf16 q/k/v/o at d = 128 take kda_prefill_tc.cu instead):
//   kda_chunk_intra  one CTA per (chunk, head), all chunks in parallel, fp32: G, Akk, Aqk
//                    with 16-token sub-block anchors, M = (I + Akk)^-1 diag(beta) by blocked
//                    forward substitution, and the scaled operands Qtil, Ktil, Kbar, e^G_C.
//   kda_scan_tc32    fp32 I/O at d = 128: one CTA per (sequence, head, 64-column half of d_v)
//                    walks the sequence's chunks on tcgen05 with the state half in TMEM,
//                    every operand a bf16 hi + lo pair (three MMAs per product):
//                    X = V - Ktil S; Delta = M X; O = Qtil S + Aqk Delta;
//                    S = e^G_C S + Kbar^T Delta.
//   kda_chunk_scan   d = 64: the same steps on the CUDA cores, one CTA per (sequence, head,
//                    32-column slice of d_v) with its state slice in registers and shared
//                    memory.
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
#include "sm100.cuh"

namespace k3 {

// kda_prefill_tc.cu: the tcgen05 form, used for bf16 q/k/v/o with d_k = d_v = 128
int run_prefill_tc(k3cuda_ctx *ctx, float *state, void *o, const void *q, const void *k,
                   const void *v, const float *gate, const float *beta, int total_tokens,
                   int n_seq, int H, float q_scale, int gate_is_log, long long nc,
                   const void *d_table, const int *d_c0, void *blocks, const GatherOut *go);
size_t prefill_tc_block_bytes();

constexpr int KC = 64;        // chunk length
constexpr int KSUB = 16;      // anchor sub-block
constexpr float kLog2eF = 1.4426950408889634f;
// largest growth factor 2^x the anchored form admits inside a sub-block (e^80, in log2 units)
constexpr float kAnchorLog2 = 80.f * kLog2eF;
constexpr int SCAN_NC = 32;   // d_v columns per scan CTA

struct ChunkDesc {
    int seq;    // sequence index
    int t0;     // first token (packed index)
    int len;    // tokens in this chunk (1..64)
    int pad;
};

// The block of one (chunk, head) for the tensor-core fp32 scan (d = 128; same size as the
// fp32 block below): every operand as a hi plane bf16(x) and a lo plane bf16(x - hi), each
// laid out as the 128-byte-swizzled shared-memory image the scan's MMAs read, so that one
// untiled bulk copy per group stages it. Byte offsets:
constexpr int W32_KQH = 0;        // [Qtil | Ktil] [128 rows][128 i], two K-blocks of [128][64]
                                  // (rows interleaved by sixteen: 32 q + l, l < 16, is Qtil
                                  // row 16 q + l; 32 q + 16 + l is Ktil row 16 q + l)
constexpr int W32_KQL = 32768;
constexpr int W32_MH = 65536;     // M = (I + Akk)^-1 diag(beta) [64 t][64 s], K-major
constexpr int W32_ML = 73728;
constexpr int W32_AH = 81920;     // Aqk [64 t][64 s], K-major
constexpr int W32_AL = 90112;
constexpr int W32_KBH = 98304;    // Kbar [64 t][128 i], two blocks [64 t][64 i] (MN-major A)
constexpr int W32_KBL = 114688;
constexpr int W32_G = 131072;     // Gamma = e^(G_C) [128] fp32
constexpr int W32_BYTES = 131584;

// hi / lo halves of x at byte `off` of the planes `hi` and `lo` of block `b`
__device__ __forceinline__ void put_split(uint8_t *b, int hi, int lo, uint32_t off, float x) {
    const __nv_bfloat16 xh = __float2bfloat16_rn(x);
    *reinterpret_cast<__nv_bfloat16 *>(b + hi + off) = xh;
    *reinterpret_cast<__nv_bfloat16 *>(b + lo + off) = __float2bfloat16_rn(x - __bfloat162float(xh));
}

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

// ---------------------------------------------------------------------------- intra
// One CTA per (chunk, head), 256 threads, two CTAs per SM. G is kept in log2 units, so every
// exponential below is one 2^x on the special-function unit. Thread (ic, grp) = (tid % DK,
// tid / DK) owns channel ic of the tokens [TG grp, TG grp + TG) and keeps their k and q in
// registers; shared memory holds G, the anchored operands of the current sub-block and Akk
// (about 101 KB at d_k = 128). Rows are padded to DK + 4 floats: the Akk / Aqk products read
// sixteen different rows of Kh at once, which then fall in different banks. Aqk goes straight
// to the workspace. (I + Akk)^-1 is formed blockwise on 16 x 16 blocks: the four diagonal
// blocks by forward substitution (one lane per column, no barrier between rows), then the
// blocks below the diagonal, one block diagonal at a time, from
// T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj. With TC32 (fp32 I/O at d = 128) the block is written
// in the tensor-core scan's layout (every operand as bf16 hi/lo planes, swizzled as its shared
// memory image); otherwise as fp32 for kda_chunk_scan.
template <typename IO, int DK, bool TC32 = false>
__global__ void __launch_bounds__(256, 2)
kda_chunk_intra(const ChunkDesc *__restrict__ chunks, const IO *__restrict__ q,
                const IO *__restrict__ k, const float *__restrict__ gate,
                const float *__restrict__ beta, float *__restrict__ ws, int H, float q_scale,
                int gate_is_log) {
    using L = PrefillLayout<DK>;
    constexpr int LP = DK + 4, NB = KC / KSUB, NG = 256 / DK, TG = KC / NG;
    extern __shared__ __align__(16) float sm[];
    float *sG = sm;                     // [KC][LP]   cumulative log decay
    float *sKh = sG + KC * LP;          // [KC][LP]   k_s e^(G_r - G_s) for the current anchor r
    float *sKa = sKh + KC * LP;         // [KSUB][LP] k_t e^(G_t - G_r)
    float *sQa = sKa + KSUB * LP;       // [KSUB][LP] q_t e^(G_t - G_r)
    float *sA = sQa + KSUB * LP;        // [KC][KC]   Akk (beta-scaled, strictly lower)
    float *sb = sA + KC * KC;           // [KC]       beta
    float *sTot = sb + KC;              // [NG][DK]   decay sum of each token group
    float *sT = sKh;                    // [KC][KC]   (I + Akk)^-1 (Kh is dead by then)
    float *sP = sKh + KC * KC;          // [NB-1][KSUB][KSUB] block products

    const ChunkDesc cd = chunks[blockIdx.x];
    const int h = blockIdx.y, tid = threadIdx.x;
    const int ic = tid % DK, grp = tid / DK, tg0 = grp * TG;
    float *out = ws + ((size_t)blockIdx.x * H + h) * L::floats;
    uint8_t *ob = reinterpret_cast<uint8_t *>(out);  // the same block, as the TC32 layout
    static_assert(!TC32 || (DK == 128 && L::floats * 4 == W32_BYTES), "TC32 block layout");

    float kr[TG], qr[TG];
    {
        // every load in flight at once: rows past the chunk's end read its last row (in
        // bounds) and are zeroed afterwards
        float gr[TG];
        {
            const size_t o0 = ((size_t)cd.t0 * H + h) * DK + ic, rs = (size_t)H * DK;
#pragma unroll
            for (int u = 0; u < TG; u++) {
                const size_t off = o0 + (size_t)min(tg0 + u, cd.len - 1) * rs;
                kr[u] = io<IO>::ld(k + off);
                qr[u] = io<IO>::ld(q + off);
                gr[u] = gate[off];
            }
#pragma unroll
            for (int u = 0; u < TG; u++) {
                const bool in = tg0 + u < cd.len;
                kr[u] = in ? kr[u] : 0.f;
                qr[u] = in ? qr[u] * q_scale : 0.f;
                // G in log2 units: every use below is 2^(difference of G values)
                gr[u] = in ? (gate_is_log ? gr[u] * kLog2eF : log2f(gr[u])) : 0.f;
            }
        }
        float acc = 0.f;
#pragma unroll
        for (int u = 0; u < TG; u++) {
            acc += gr[u];
            gr[u] = acc;
        }
        sTot[grp * DK + ic] = acc;
        if (tid < KC) sb[tid] = tid < cd.len ? beta[(size_t)(cd.t0 + tid) * H + h] : 0.f;
        __syncthreads();
        float base = 0.f;
        for (int g2 = 0; g2 < grp; g2++) base += sTot[g2 * DK + ic];
#pragma unroll
        for (int u = 0; u < TG; u++) sG[(tg0 + u) * LP + ic] = gr[u] + base;
    }
    __syncthreads();

    // scaled operands for the scan (full-chunk anchor at the chunk start)
    {
        const float GC = sG[(KC - 1) * LP + ic];
#pragma unroll
        for (int u = 0; u < TG; u++) {
            const int t = tg0 + u;
            const float G = sG[t * LP + ic];
            const float eg = sm100::ex2_approx(G);
            if constexpr (TC32) {
                // Qtil row t at A row 32 (t / 16) + t % 16, Ktil row t sixteen rows after it
                const int rq = 32 * (t >> 4) + (t & 15);
                const uint32_t kq = (ic >> 6) * 16384 + sm100::swz_elem(rq, ic & 63);
                put_split(ob, W32_KQH, W32_KQL, kq, qr[u] * eg);
                put_split(ob, W32_KQH, W32_KQL, kq + 16 * 128, kr[u] * eg);
                put_split(ob, W32_KBH, W32_KBL, (ic >> 6) * 8192 + sm100::swz_elem(t, ic & 63),
                          kr[u] * sm100::ex2_approx(GC - G));
            } else {
                out[L::qt + t * DK + ic] = qr[u] * eg;
                out[L::kt + t * DK + ic] = kr[u] * eg;
                out[L::kb + t * DK + ic] = kr[u] * sm100::ex2_approx(GC - G);
            }
        }
        if (tid < DK) {
            if constexpr (TC32)
                reinterpret_cast<float *>(ob + W32_G)[tid] = sm100::ex2_approx(GC);
            else
                out[L::gc + tid] = sm100::ex2_approx(GC);
        }
    }

    // Akk / Aqk, one 16-row sub-block at a time; thread (tl, ss) = (tid / 16, tid % 16) forms
    // row r0 + tl against the columns ss + 16 m, m = 0..a
#pragma unroll
    for (int a = 0; a < NB; a++) {
        const int r0 = a * KSUB, ncol = r0 + KSUB;
        const float Gr = sG[r0 * LP + ic];
        int big = 0;
#pragma unroll
        for (int u = 0; u < TG; u++) {
            const int s = tg0 + u;
            if (s < ncol) {
                const float Gs = sG[s * LP + ic];
                const float ex = Gr - Gs;
                big |= ex > kAnchorLog2;
                sKh[s * LP + ic] = kr[u] * sm100::ex2_approx(fminf(ex, kAnchorLog2));
                if (s >= r0) {
                    const float f = sm100::ex2_approx(Gs - Gr);
                    sKa[(s - r0) * LP + ic] = kr[u] * f;
                    sQa[(s - r0) * LP + ic] = qr[u] * f;
                }
            }
        }
        big = __syncthreads_or(big);
        const int tl = tid / 16, ss = tid % 16, t = r0 + tl;
        float akk[NB], aqk[NB];
#pragma unroll
        for (int m = 0; m < NB; m++) akk[m] = aqk[m] = 0.f;
#pragma unroll 2
        for (int i = 0; i < DK; i += 4) {
            const float4 ka = *reinterpret_cast<const float4 *>(sKa + tl * LP + i);
            const float4 qa = *reinterpret_cast<const float4 *>(sQa + tl * LP + i);
#pragma unroll
            for (int m = 0; m <= a; m++) {
                const float4 kh = *reinterpret_cast<const float4 *>(sKh + (ss + 16 * m) * LP + i);
                akk[m] += ka.x * kh.x;
                akk[m] += ka.y * kh.y;
                akk[m] += ka.z * kh.z;
                akk[m] += ka.w * kh.w;
                aqk[m] += qa.x * kh.x;
                aqk[m] += qa.y * kh.y;
                aqk[m] += qa.z * kh.z;
                aqk[m] += qa.w * kh.w;
            }
        }
#pragma unroll
        for (int m = 0; m < NB; m++) {
            const int s = ss + 16 * m;
            float vk = 0.f, vq = 0.f;
            if (m <= a && s <= t) {
                vk = akk[m];
                vq = aqk[m];
                if (big && s >= r0) {
                    // exact path from the inputs (k and q are zero past the chunk's tokens)
                    vk = vq = 0.f;
                    if (t < cd.len) {
                        const size_t ot = ((size_t)(cd.t0 + t) * H + h) * DK;
                        const size_t os = ((size_t)(cd.t0 + s) * H + h) * DK;
                        for (int i = 0; i < DK; i++) {
                            const float f =
                                sm100::ex2_approx(sG[t * LP + i] - sG[s * LP + i]) *
                                io<IO>::ld(k + os + i);
                            vk += io<IO>::ld(k + ot + i) * f;
                            vq += io<IO>::ld(q + ot + i) * q_scale * f;
                        }
                    }
                }
            }
            sA[t * KC + s] = s < t ? sb[t] * vk : 0.f;
            if constexpr (TC32)
                put_split(ob, W32_AH, W32_AL, sm100::swz_elem(t, s), vq);
            else
                out[L::aqk + t * KC + s] = vq;
        }
        __syncthreads();
    }

    // diagonal blocks of T = (I + Akk)^-1: warp d, lane c < 16 owns column 16 d + c of block d
    if (tid < 32 * NB && tid % 32 < KSUB) {
        const int d = tid / 32, c = tid % 32, b0 = d * KSUB;
        float col[KSUB];
#pragma unroll
        for (int r = 0; r < KSUB; r++) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < r; j++)
                if (j >= c) acc += sA[(b0 + r) * KC + b0 + j] * col[j];
            col[r] = r == c ? 1.f : (r > c ? -acc : 0.f);
        }
#pragma unroll
        for (int r = 0; r < KSUB; r++) sT[(b0 + r) * KC + b0 + c] = col[r];
    }
    __syncthreads();
    // blocks below the diagonal, one block diagonal (delta = i - j) at a time
    for (int delta = 1; delta < NB; delta++) {
        const int nblk = NB - delta;
        for (int e = tid; e < nblk * KSUB * KSUB; e += 256) {
            const int bj = e / (KSUB * KSUB), r = (e / KSUB) % KSUB, c = e % KSUB;
            const int bi = bj + delta;
            float acc = 0.f;
            for (int x = bj * KSUB; x < bi * KSUB; x++)
                acc += sA[(bi * KSUB + r) * KC + x] * sT[x * KC + bj * KSUB + c];
            sP[e] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nblk * KSUB * KSUB; e += 256) {
            const int bj = e / (KSUB * KSUB), r = (e / KSUB) % KSUB, c = e % KSUB;
            const int bi = bj + delta;
            const float *P = sP + bj * KSUB * KSUB;
            float acc = 0.f;
#pragma unroll
            for (int x = 0; x < KSUB; x++)
                acc += sT[(bi * KSUB + r) * KC + bi * KSUB + x] * P[x * KSUB + c];
            sT[(bi * KSUB + r) * KC + bj * KSUB + c] = -acc;
        }
        __syncthreads();
    }
    // M = T diag(beta), zero above the diagonal blocks
    for (int e = tid; e < KC * KC; e += 256) {
        const int t = e / KC, s = e % KC;
        const float mv = t / KSUB < s / KSUB ? 0.f : sT[e] * sb[s];
        if constexpr (TC32)
            put_split(ob, W32_MH, W32_ML, sm100::swz_elem(t, s), mv);
        else
            out[L::m + e] = mv;
    }
}

// ----------------------------------------------------------------------------- scan
// 16-byte asynchronous copies global -> shared (cp.async): the next chunk's operands stream in
// while the current chunk computes. A wait_group waits only for this thread's own copies, which
// complete without any condition on other threads, so no wait here needs a bound.
__device__ __forceinline__ void cp_async16(float *dst, const float *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// rows x cols floats (row stride cols in global) into shared rows of stride ld, 256 threads
template <int ROWS, int COLS, int LD>
__device__ __forceinline__ void stage_rows(float *dst, const float *src, int tid) {
    constexpr int Q = COLS / 4;
#pragma unroll
    for (int e = tid; e < ROWS * Q; e += 256) {
        const int r = e / Q, c = e - r * Q;
        cp_async16(dst + r * LD + 4 * c, src + r * COLS + 4 * c);
    }
}

__device__ __forceinline__ void fma4(float (&acc)[4], float a, const float4 &b) {
    acc[0] += a * b.x;
    acc[1] += a * b.y;
    acc[2] += a * b.z;
    acc[3] += a * b.w;
}

template <typename IO>
__device__ __forceinline__ void load4(float (&x)[4], const IO *p) {
#pragma unroll
    for (int u = 0; u < 4; u++) x[u] = io<IO>::ld(p + u);
}

// One CTA per (sequence, head, 32-column slice of d_v), 256 threads. Thread (tx, ty) =
// (tid % 8, tid / 8) owns columns 4tx..4tx+3 of the slice, the token pair (ty, 63 - ty) in the
// token phases (the pair's triangular sums in M X and Aqk Delta have 65 terms for every ty,
// so the eight warps finish those phases together) and state rows (DK/32) ty .. of the update.
// Operands: Qtil / Ktil rows padded to DK + 4 floats and M / Aqk rows to 68, so the four rows
// a warp reads at once fall in different banks. Per chunk the copies are three groups, each
// issued as soon as the phase that read the previous chunk's copy has ended:
//   G1 = Ktil, Qtil (read in phase A)   G2 = M (phase B)   G3 = Aqk, Kbar, e^G_C (phase C/D)
// Sums run in the recurrence's order (over i, then over s, ascending), as in the oracle.
template <typename IO, int DK>
__global__ void __launch_bounds__(256, 1)
kda_chunk_scan(const ChunkDesc *__restrict__ chunks, const int *__restrict__ seq_chunk0,
               const int *__restrict__ seq_order, const IO *__restrict__ v,
               const float *__restrict__ ws, float *__restrict__ state, IO *__restrict__ o,
               int H) {
    using L = PrefillLayout<DK>;
    constexpr int DV = DK, NT = DV / SCAN_NC, LK = DK + 4, LM = KC + 4, RS = DK / 32;
    static_assert(RS == 2 || RS == 4, "state rows per thread");
    extern __shared__ __align__(16) float sm[];
    float *sKt = sm;                    // [KC][LK]  Ktil
    float *sQt = sKt + KC * LK;         // [KC][LK]  Qtil
    float *sKb = sQt + KC * LK;         // [KC][DK]  Kbar
    float *sM = sKb + KC * DK;          // [KC][LM]  M = (I + Akk)^-1 diag(beta)
    float *sAq = sM + KC * LM;          // [KC][LM]  Aqk
    float *sGc = sAq + KC * LM;         // [DK]      e^G_C
    float *sS = sGc + DK;               // [DK][SCAN_NC]  state slice
    float *sX = sS + DK * SCAN_NC;      // [KC][SCAN_NC]  V - Ktil S
    float *sD = sX + KC * SCAN_NC;      // [KC][SCAN_NC]  Delta

    const int tile = blockIdx.x % NT;
    const int h = (blockIdx.x / NT) % H;
    const int n = seq_order[blockIdx.x / (NT * H)];
    const int tid = threadIdx.x, w = tid / 32, tx = tid % 8, ty = tid / 8;
    const int ta = ty, tb = KC - 1 - ty, cj = 4 * tx, col0 = tile * SCAN_NC + cj;
    const int c0 = seq_chunk0[n], c1 = seq_chunk0[n + 1];
    float *Sg = state ? state + ((size_t)n * H + h) * DK * DV : nullptr;

    float sreg[RS][4];
#pragma unroll
    for (int r = 0; r < RS; r++) {
        const int i = RS * ty + r;
#pragma unroll
        for (int u = 0; u < 4; u++) sreg[r][u] = Sg ? Sg[(size_t)i * DV + col0 + u] : 0.f;
        *reinterpret_cast<float4 *>(sS + i * SCAN_NC + cj) =
            make_float4(sreg[r][0], sreg[r][1], sreg[r][2], sreg[r][3]);
    }

    auto block = [&](int c) { return ws + ((size_t)c * H + h) * L::floats; };
    auto issue_g1 = [&](int c) {
        const float *b = block(c);
        stage_rows<KC, DK, LK>(sKt, b + L::kt, tid);
        stage_rows<KC, DK, LK>(sQt, b + L::qt, tid);
    };
    auto issue_g2 = [&](int c) { stage_rows<KC, KC, LM>(sM, block(c) + L::m, tid); };
    auto issue_g3 = [&](int c) {
        const float *b = block(c);
        stage_rows<KC, KC, LM>(sAq, b + L::aqk, tid);
        stage_rows<KC, DK, DK>(sKb, b + L::kb, tid);
        stage_rows<1, DK, DK>(sGc, b + L::gc, tid);
    };
    if (c0 < c1) issue_g1(c0);
    cp_async_commit();
    if (c0 < c1) issue_g2(c0);
    cp_async_commit();

    for (int c = c0; c < c1; c++) {
        const ChunkDesc cd = chunks[c];
        float xa[4] = {0.f, 0.f, 0.f, 0.f}, xb[4] = {0.f, 0.f, 0.f, 0.f};
        if (ta < cd.len) load4<IO>(xa, v + ((size_t)(cd.t0 + ta) * H + h) * DV + col0);
        if (tb < cd.len) load4<IO>(xb, v + ((size_t)(cd.t0 + tb) * H + h) * DV + col0);
        cp_async_wait<1>();  // G1(c)
        __syncthreads();     // ... for every thread; the previous chunk's phase C/D is over
        issue_g3(c);
        cp_async_commit();

        // phase A: Ktil S and Qtil S for tokens ta and tb
        float ka[4] = {0.f, 0.f, 0.f, 0.f}, kb[4] = {0.f, 0.f, 0.f, 0.f};
        float qa[4] = {0.f, 0.f, 0.f, 0.f}, qb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int i = 0; i < DK; i += 4) {
            const float4 Ka = *reinterpret_cast<const float4 *>(sKt + ta * LK + i);
            const float4 Kb = *reinterpret_cast<const float4 *>(sKt + tb * LK + i);
            const float4 Qa = *reinterpret_cast<const float4 *>(sQt + ta * LK + i);
            const float4 Qb = *reinterpret_cast<const float4 *>(sQt + tb * LK + i);
            const float ka_[4] = {Ka.x, Ka.y, Ka.z, Ka.w}, kb_[4] = {Kb.x, Kb.y, Kb.z, Kb.w};
            const float qa_[4] = {Qa.x, Qa.y, Qa.z, Qa.w}, qb_[4] = {Qb.x, Qb.y, Qb.z, Qb.w};
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float4 s = *reinterpret_cast<const float4 *>(sS + (i + u) * SCAN_NC + cj);
                fma4(ka, ka_[u], s);
                fma4(kb, kb_[u], s);
                fma4(qa, qa_[u], s);
                fma4(qb, qb_[u], s);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            xa[u] -= ka[u];
            xb[u] -= kb[u];
        }
        *reinterpret_cast<float4 *>(sX + ta * SCAN_NC + cj) = make_float4(xa[0], xa[1], xa[2], xa[3]);
        *reinterpret_cast<float4 *>(sX + tb * SCAN_NC + cj) = make_float4(xb[0], xb[1], xb[2], xb[3]);
        cp_async_wait<1>();  // G2(c)
        __syncthreads();
        if (c + 1 < c1) issue_g1(c + 1);
        cp_async_commit();

        // phase B: Delta = M X; M is lower triangular, so token t sums s = 0..t (the entries
        // above the diagonal are zeros and the last group of four stops at t's group)
        float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < KC / 4 - w; q++) {
            const int s = 4 * q;
            const float4 Mb = *reinterpret_cast<const float4 *>(sM + tb * LM + s);
            const float mb_[4] = {Mb.x, Mb.y, Mb.z, Mb.w};
            float4 x[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                x[u] = *reinterpret_cast<const float4 *>(sX + (s + u) * SCAN_NC + cj);
#pragma unroll
            for (int u = 0; u < 4; u++) fma4(db, mb_[u], x[u]);
            if (q <= w) {
                const float4 Ma = *reinterpret_cast<const float4 *>(sM + ta * LM + s);
                const float ma_[4] = {Ma.x, Ma.y, Ma.z, Ma.w};
#pragma unroll
                for (int u = 0; u < 4; u++) fma4(da, ma_[u], x[u]);
            }
        }
        *reinterpret_cast<float4 *>(sD + ta * SCAN_NC + cj) = make_float4(da[0], da[1], da[2], da[3]);
        *reinterpret_cast<float4 *>(sD + tb * SCAN_NC + cj) = make_float4(db[0], db[1], db[2], db[3]);
        cp_async_wait<1>();  // G3(c)
        __syncthreads();
        if (c + 1 < c1) issue_g2(c + 1);
        cp_async_commit();

        // phase C: O = Qtil S + Aqk Delta (Aqk lower triangular with its diagonal)
        for (int q = 0; q < KC / 4 - w; q++) {
            const int s = 4 * q;
            const float4 Ab = *reinterpret_cast<const float4 *>(sAq + tb * LM + s);
            const float ab_[4] = {Ab.x, Ab.y, Ab.z, Ab.w};
            float4 d[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                d[u] = *reinterpret_cast<const float4 *>(sD + (s + u) * SCAN_NC + cj);
#pragma unroll
            for (int u = 0; u < 4; u++) fma4(qb, ab_[u], d[u]);
            if (q <= w) {
                const float4 Aa = *reinterpret_cast<const float4 *>(sAq + ta * LM + s);
                const float aa_[4] = {Aa.x, Aa.y, Aa.z, Aa.w};
#pragma unroll
                for (int u = 0; u < 4; u++) fma4(qa, aa_[u], d[u]);
            }
        }
        if (ta < cd.len) {
            IO *op = o + ((size_t)(cd.t0 + ta) * H + h) * DV + col0;
#pragma unroll
            for (int u = 0; u < 4; u++) io<IO>::st(op + u, qa[u]);
        }
        if (tb < cd.len) {
            IO *op = o + ((size_t)(cd.t0 + tb) * H + h) * DV + col0;
#pragma unroll
            for (int u = 0; u < 4; u++) io<IO>::st(op + u, qb[u]);
        }

        // phase D: S = e^G_C S + Kbar^T Delta for state rows RS ty .. RS ty + RS - 1
#pragma unroll
        for (int r = 0; r < RS; r++) {
            const float g = sGc[RS * ty + r];
#pragma unroll
            for (int u = 0; u < 4; u++) sreg[r][u] = g * sreg[r][u];
        }
#pragma unroll 4
        for (int s = 0; s < KC; s++) {
            const float4 d = *reinterpret_cast<const float4 *>(sD + s * SCAN_NC + cj);
            float kbar[RS];
            if constexpr (RS == 4) {
                const float4 k4 = *reinterpret_cast<const float4 *>(sKb + s * DK + 4 * ty);
                kbar[0] = k4.x, kbar[1] = k4.y, kbar[2] = k4.z, kbar[3] = k4.w;
            } else {
                const float2 k2 = *reinterpret_cast<const float2 *>(sKb + s * DK + 2 * ty);
                kbar[0] = k2.x, kbar[1] = k2.y;
            }
#pragma unroll
            for (int r = 0; r < RS; r++) fma4(sreg[r], kbar[r], d);
        }
#pragma unroll
        for (int r = 0; r < RS; r++)
            *reinterpret_cast<float4 *>(sS + (RS * ty + r) * SCAN_NC + cj) =
                make_float4(sreg[r][0], sreg[r][1], sreg[r][2], sreg[r][3]);
    }
    cp_async_wait<0>();
    if (Sg)
#pragma unroll
        for (int r = 0; r < RS; r++)
#pragma unroll
            for (int u = 0; u < 4; u++)
                Sg[(size_t)(RS * ty + r) * DV + col0 + u] = sreg[r][u];
}

// ------------------------------------------------------------ scan on tcgen05 (fp32 I/O)
// Shared-memory plan of kda_scan_tc32 (bytes from a 1024-aligned base). The operand groups
// keep the offsets of the workspace block, so each is one bulk copy.
struct Scan32 {
    static constexpr int KQ = W32_KQH, KQ_BYTES = 65536;   // [Qtil | Ktil] hi, lo
    static constexpr int M = W32_MH, M_BYTES = 16384;      // M hi, lo
    static constexpr int KA = W32_AH, KA_BYTES = 49152;    // Aqk hi, lo; Kbar hi, lo
    static constexpr int S16H = 131072, S16L = 147456;     // state [128 i][64 j], MN-major
    static constexpr int XH = 163840, XL = 172032;         // X = V - Ktil S [64 s][64 j]
    static constexpr int DH = 180224, DL = 188416;         // Delta = M X [64 s][64 j]
    static constexpr int BYTES = 196608, SMEM = BYTES + 1024;
    static constexpr uint32_t TM_Y = 0, TM_D = 128, TM_S = 192, TM_COLS = 256;
    static constexpr int THREADS = 320;                    // 8 compute warps, producer, MMA
};
static_assert(Scan32::SMEM <= 232448, "tc32 scan shared memory");
static_assert(W32_KQL == W32_KQH + 32768 && W32_AH + Scan32::KA_BYTES == W32_G,
              "operand groups are contiguous in the workspace block");

__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

template <bool VEC>
__device__ __forceinline__ void ld_row32(float *dst, const float *src) {
    if constexpr (VEC) {
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
            const float4 x = *reinterpret_cast<const float4 *>(src + c);
            dst[c] = x.x, dst[c + 1] = x.y, dst[c + 2] = x.z, dst[c + 3] = x.w;
        }
    } else {
#pragma unroll
        for (int c = 0; c < 32; c++) dst[c] = src[c];
    }
}
template <bool VEC>
__device__ __forceinline__ void st_row32(float *dst, const float *src) {
    if constexpr (VEC) {
#pragma unroll
        for (int c = 0; c < 32; c += 4)
            *reinterpret_cast<float4 *>(dst + c) =
                make_float4(src[c], src[c + 1], src[c + 2], src[c + 3]);
    } else {
#pragma unroll
        for (int c = 0; c < 32; c++) dst[c] = src[c];
    }
}
// bf16 hi and lo halves of 32 values into columns [32 hf, 32 hf + 32) of row r of two
// MN-major [rows][64] tiles
__device__ __forceinline__ void put_half_split(uint8_t *hi, uint8_t *lo, int r, int hf,
                                               const float *x) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
        float h[8], l[8];
        const uint4 ph = sm100::pack_bf8(x + 8 * c);
        sm100::unpack_bf8(ph, h);
#pragma unroll
        for (int u = 0; u < 8; u++) l[u] = x[8 * c + u] - h[u];
        sm100::st16s(hi + sm100::swz(r, 4 * hf + c), ph);
        sm100::st16s(lo + sm100::swz(r, 4 * hf + c), sm100::pack_bf8(l));
    }
}

// Chunk scan in the direct form on tcgen05, for fp32 q/k/v/o at d_k = d_v = 128, with
// fp32-level products: every operand is a bf16 pair hi + lo and every product is three MMAs
// (hi.hi + hi.lo + lo.hi, fp32 accumulation in TMEM), which leaves about 2^-16 relative error
// per product instead of bf16's 2^-8. One CTA per (sequence, head, 64-column half of d_v);
// the fp32 state half lives in TMEM. Per chunk:
//   Y  = [Qtil | Ktil] S16        (M=128; the A rows interleave by sixteen: row 32 q + l is
//                                 Qtil row 16 q + l for l < 16 and Ktil row 16 q + l - 16
//                                 otherwise, so every TMEM lane quarter holds 16 rows of each)
//   X  = V - (Ktil S)             lanes 16-31 of every quarter, bf16 hi/lo to shared memory
//   D  = M X                      (M=64)
//   S' = Gamma S + Kbar^T D       (M=128, into the state accumulator, already scaled)
//   O  = Qtil S + Aqk D           (M=64 into Y's columns: an M=64 accumulator's row 16 q + l
//                                 is lane 32 q + l, exactly where Y holds Qtil S)
// then S' is copied to S16 (hi/lo) and scaled by the next Gamma in TMEM. Warps 0-7 compute:
// warp w reads lane quarter w % 4, columns [32 (w / 4), +32); warp 8: bulk-copy producer;
// warp 9: TMEM allocation and MMA issue. Y is double-buffered in TMEM so that a chunk's
// outputs are read while the next chunk runs.
template <bool VEC>
__global__ void __launch_bounds__(Scan32::THREADS, 1)
kda_scan_tc32(const ChunkDesc *__restrict__ chunks, const int *__restrict__ seq_chunk0,
              const int *__restrict__ seq_order, const uint8_t *__restrict__ ws,
              const float *__restrict__ v, float *__restrict__ state, float *__restrict__ o,
              int H, unsigned *__restrict__ err) {
    using namespace sm100;
    using C = Scan32;
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t kq_full, kq_empty, m_full, m_empty, ka_full, ka_empty;
    __shared__ uint64_t y_done, x_ready, dx_done, d_ready, s_done, o_done, s16_ready, mma_fin;
    __shared__ uint32_t tslot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int half = blockIdx.x & 1, h = (blockIdx.x >> 1) % H;
    const int n = seq_order[blockIdx.x / (2 * H)];
    const int c0 = seq_chunk0[n], nc = seq_chunk0[n + 1] - c0;
    const int col0 = 64 * half;
    constexpr uint32_t NCOMP = 256;
    auto block = [&](int j) { return ws + ((size_t)(c0 + j) * H + h) * W32_BYTES; };

    if (tid == 0) {
        mbar_init(&kq_full, 1);
        mbar_init(&kq_empty, 1);
        mbar_init(&m_full, 1);
        mbar_init(&m_empty, 1);
        mbar_init(&ka_full, 1);
        mbar_init(&ka_empty, 1);
        mbar_init(&y_done, 1);
        mbar_init(&x_ready, NCOMP);
        mbar_init(&dx_done, 1);
        mbar_init(&d_ready, NCOMP);
        mbar_init(&s_done, 1);
        mbar_init(&o_done, 1);
        mbar_init(&s16_ready, NCOMP);
        mbar_init(&mma_fin, 1);
        fence_barrier_init();
    }
    if (warp == 9) tmem_alloc(&tslot, C::TM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tslot;

    if (warp == 8) {
        if (lane == 0) {
            int last_kq = -1, last_m = -1, last_ka = -1;
            for (int j = 0; j < nc; j++) {
                const uint8_t *b = block(j);
                const uint32_t pe = (j - 1) & 1;
                if (j > 0 && !mbar_wait(&kq_empty, pe, err, 0x701)) break;
                mbar_expect_tx(&kq_full, C::KQ_BYTES);
                bulk_load(sm + C::KQ, b + W32_KQH, C::KQ_BYTES, &kq_full);
                last_kq = j;
                if (j > 0 && !mbar_wait(&m_empty, pe, err, 0x702)) break;
                mbar_expect_tx(&m_full, C::M_BYTES);
                bulk_load(sm + C::M, b + W32_MH, C::M_BYTES, &m_full);
                last_m = j;
                if (j > 0 && !mbar_wait(&ka_empty, pe, err, 0x703)) break;
                // and after this chunk's Y products, so that the copy does not compete with
                // them for shared memory (it is first read by the chunk's state update)
                if (!mbar_wait(&kq_empty, j & 1, err, 0x70e)) break;
                mbar_expect_tx(&ka_full, C::KA_BYTES);
                bulk_load(sm + C::KA, b + W32_AH, C::KA_BYTES, &ka_full);
                last_ka = j;
            }
            // copies still in flight are waited for (bounded) before the CTA may exit
            if (last_kq >= 0) mbar_wait_quiet(&kq_full, last_kq & 1);
            if (last_m >= 0) mbar_wait_quiet(&m_full, last_m & 1);
            if (last_ka >= 0) mbar_wait_quiet(&ka_full, last_ka & 1);
        }
    } else if (warp == 9) {
        if (lane == 0) {
            constexpr uint32_t id_y = idesc_f16(128, 64, false, true);
            constexpr uint32_t id_m = idesc_f16(64, 64, false, true);
            constexpr uint32_t id_s = idesc_f16(128, 64, true, true);
            const uint64_t dk = sdesc_kmajor(smem_u32(sm));
            const uint64_t d8 = sdesc_mnmajor(smem_u32(sm), 8192);
            const uint64_t d16 = sdesc_mnmajor(smem_u32(sm), 16384);
            bool issued = false;
            for (int j = 0; j < nc; j++) {
                const uint32_t par = j & 1, yb = tb + C::TM_Y + 64 * (j & 1);
                // Y = [Qtil | Ktil] . S16
                if (!mbar_wait(&kq_full, par, err, 0x704)) break;
                if (!mbar_wait(&s16_ready, par, err, 0x705)) break;
                tc_fence_after();
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    const int a = C::KQ + (p == 2 ? 32768 : 0), b = p == 1 ? C::S16L : C::S16H;
#pragma unroll
                    for (int ks = 0; ks < 8; ks++)
                        mma_bf16_ss(yb, dk + ((a + (ks >> 2) * 16384 + (ks & 3) * 32) >> 4),
                                    d16 + ((b + ks * 2048) >> 4), id_y, (p | ks) ? 1u : 0u);
                }
                issued = true;
                mma_commit(&y_done);
                mma_commit(&kq_empty);
                // D = M . X
                if (!mbar_wait(&m_full, par, err, 0x706)) break;
                if (!mbar_wait(&x_ready, par, err, 0x707)) break;
                tc_fence_after();
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    const int a = p == 2 ? W32_ML : W32_MH, b = p == 1 ? C::XL : C::XH;
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        mma_bf16_ss(tb + C::TM_D, dk + ((a + ks * 32) >> 4),
                                    d8 + ((b + ks * 2048) >> 4), id_m, (p | ks) ? 1u : 0u);
                }
                mma_commit(&dx_done);
                mma_commit(&m_empty);
                // S += Kbar^T . D, then O (the Qtil rows of Y) += Aqk . D
                if (!mbar_wait(&ka_full, par, err, 0x708)) break;
                if (!mbar_wait(&d_ready, par, err, 0x709)) break;
                tc_fence_after();
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    const int a = p == 2 ? W32_KBL : W32_KBH, b = p == 1 ? C::DL : C::DH;
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        mma_bf16_ss(tb + C::TM_S, d8 + ((a + ks * 2048) >> 4),
                                    d8 + ((b + ks * 2048) >> 4), id_s, 1u);
                }
                mma_commit(&s_done);
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    const int a = p == 2 ? W32_AL : W32_AH, b = p == 1 ? C::DL : C::DH;
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        mma_bf16_ss(yb, dk + ((a + ks * 32) >> 4), d8 + ((b + ks * 2048) >> 4),
                                    id_m, 1u);
                }
                mma_commit(&o_done);
                mma_commit(&ka_empty);
            }
            // every MMA issued (an aborted loop included) completes before TMEM is freed
            if (issued) {
                mma_commit(&mma_fin);
                mbar_wait_quiet(&mma_fin, 0);
            }
        }
    } else if (nc > 0) {
        // ----------------------------------------------------------- compute warps
        const int q = warp & 3, hf = warp >> 2;          // lane quarter, column half
        const int i = 32 * q + lane;                     // TMEM lane: state row i
        const int r16 = 16 * q + (lane & 15);            // token row of this lane's Y / D / O
        const uint32_t lq = ((uint32_t)(32 * q) << 16) + 32 * hf;
        float *Sg = state ? state + (((size_t)n * H + h) * 128 + i) * 128 + col0 + 32 * hf
                          : nullptr;
        auto gamma = [&](int jj) {
            return jj < nc ? reinterpret_cast<const float *>(block(jj) + W32_G)[i] : 0.f;
        };
        float s[32];
        auto tmem_row = [&](uint32_t col, float *dst) {
            tmem_ld32(tb + lq + col, dst);
            tmem_wait_ld();
        };
        // S16 <- S (hi, lo); TMEM state <- gam * S
        auto publish = [&](float gam) {
            put_half_split(sm + C::S16H, sm + C::S16L, i, hf, s);
#pragma unroll
            for (int c = 0; c < 32; c += 16) {
                float x[16];
#pragma unroll
                for (int u = 0; u < 16; u++) x[u] = s[c + u] * gam;
                tmem_st16(tb + lq + C::TM_S + c, x);
            }
            tmem_wait_st();
            fence_async_shared();
            tc_fence_before();
            mbar_arrive(&s16_ready);
        };
        if (Sg) {
            ld_row32<VEC>(s, Sg);
        } else {
#pragma unroll
            for (int c = 0; c < 32; c++) s[c] = 0.f;
        }
        publish(gamma(0));
        float gam1 = gamma(1), gam2 = gamma(2);
        const bool krow = lane >= 16;  // this lane's Y row is Ktil S (else Qtil S)
        auto vrow = [&](const ChunkDesc &c) {
            return v + ((size_t)(c.t0 + r16) * H + h) * 128 + col0 + 32 * hf;
        };
        // the chunk table runs one chunk ahead and V two (into L2), so that the V rows a
        // chunk subtracts are on chip when its Y is ready
        ChunkDesc cd_next = chunks[c0];
        if (krow && nc > 1) {
            const ChunkDesc c1 = chunks[c0 + 1];
            if (r16 < c1.len) prefetch_l2(vrow(c1));
        }
        bool ok = true;
        for (int j = 0; j < nc && ok; j++) {
            const ChunkDesc cd = cd_next;
            if (j + 1 < nc) cd_next = chunks[c0 + j + 1];
            const uint32_t par = j & 1, yb = C::TM_Y + 64 * (j & 1);
            // X = V - Ktil S; V is loaded before the wait
            float x[32];
            if (krow) {
                if (r16 < cd.len) {
                    ld_row32<VEC>(x, vrow(cd));
                } else {
#pragma unroll
                    for (int c = 0; c < 32; c++) x[c] = 0.f;
                }
                if (j + 2 < nc) {
                    const ChunkDesc c2 = chunks[c0 + j + 2];
                    if (r16 < c2.len) prefetch_l2(vrow(c2));
                }
            }
            if (!(ok = warp_wait_all(&y_done, par, err, 0x70a))) break;
            tc_fence_after();
            {
                float y[32];
                tmem_row(yb, y);
                if (krow) {
#pragma unroll
                    for (int c = 0; c < 32; c++) x[c] -= y[c];
                    put_half_split(sm + C::XH, sm + C::XL, r16, hf, x);
                }
            }
            fence_async_shared();
            tc_fence_before();
            mbar_arrive(&x_ready);
            // D rows to shared memory (row 16 q + lane on lanes 0-15)
            if (!(ok = warp_wait_all(&dx_done, par, err, 0x70b))) break;
            tc_fence_after();
            {
                float dd[32];
                tmem_row(C::TM_D, dd);
                if (!krow) put_half_split(sm + C::DH, sm + C::DL, r16, hf, dd);
            }
            fence_async_shared();
            tc_fence_before();
            mbar_arrive(&d_ready);
            // the updated state: next chunk's S16 and Gamma-scaled TMEM copy, or the result
            if (!(ok = warp_wait_all(&s_done, par, err, 0x70c))) break;
            tc_fence_after();
            tmem_row(C::TM_S, s);
            if (j + 1 < nc) {
                publish(gam1);
                gam1 = gam2;
                gam2 = gamma(j + 3);
            } else if (Sg) {
                st_row32<VEC>(Sg, s);
            }
            // outputs of the chunk (the Qtil rows of Y, lanes 0-15)
            if (!(ok = warp_wait_all(&o_done, par, err, 0x70d))) break;
            tc_fence_after();
            {
                float y[32];
                tmem_row(yb, y);
                if (!krow && r16 < cd.len)
                    st_row32<VEC>(o + ((size_t)(cd.t0 + r16) * H + h) * 128 + col0 + 32 * hf, y);
            }
            tc_fence_before();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        __syncwarp();
        tmem_dealloc(tb, C::TM_COLS);
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
    const size_t smem1 = ((size_t)2 * KC * (DK + 4) + 2 * KSUB * (DK + 4) + KC * KC + KC + 256) *
                         sizeof(float);
    if constexpr (std::is_same<IO, __nv_bfloat16>::value && DK == 128) {
        // bf16 operands on the tensor cores (every operand bf16, accumulation fp32)
        (void)smem1;
        if (nc == 0) return K3CUDA_OK;
        return run_prefill_tc(ctx, state, o, q, k, v, gate, beta, cu[n_seq], n_seq, H, q_scale,
                              gate_is_log, nc, d_table, d_c0, blocks, go);
    } else if constexpr (std::is_same<IO, float>::value && DK == 128) {
        // fp32 q/k/v/o at d = 128: fp32 intra-chunk kernel writing bf16 hi/lo operands, scan on
        // the tensor cores
        if (nc == 0) return K3CUDA_OK;
        if (int rc_ = set_smem(kda_chunk_intra<float, 128, true>, (int)smem1)) return rc_;
        kda_chunk_intra<float, 128, true><<<dim3((unsigned)nc, (unsigned)H), 256, smem1,
                                            ctx->stream>>>(d_table, (const float *)q,
                                                           (const float *)k, gate, beta, blocks,
                                                           H, q_scale, gate_is_log);
        if (int rc_ = after_launch(ctx, "kda_chunk_intra")) return rc_;
        const bool vec = aligned(v, 16) && aligned(o, 16) && (!state || aligned(state, 16));
        const unsigned nblk32 = (unsigned)((long long)n_seq * H * 2);
        auto launch = [&](auto kern) {
            if (int rc_ = set_smem(kern, Scan32::SMEM)) return rc_;
            kern<<<nblk32, Scan32::THREADS, Scan32::SMEM, ctx->stream>>>(
                d_table, d_c0, d_c0 + n_seq + 1, (const uint8_t *)blocks, (const float *)v, state,
                (float *)o, H, ctx->err_word);
            return after_launch(ctx, "kda_scan_tc32");
        };
        return vec ? launch(kda_scan_tc32<true>) : launch(kda_scan_tc32<false>);
    } else {
        // d = 64: both kernels on the CUDA cores
        if (nc > 0) {
            if (int rc_ = set_smem(kda_chunk_intra<IO, DK>, (int)smem1)) return rc_;
            dim3 g1((unsigned)nc, (unsigned)H);
            kda_chunk_intra<IO, DK><<<g1, 256, smem1, ctx->stream>>>(
                d_table, (const IO *)q, (const IO *)k, gate, beta, blocks, H, q_scale, gate_is_log);
            int rc = after_launch(ctx, "kda_chunk_intra");
            if (rc) return rc;
        }
        const size_t smem2 = ((size_t)2 * KC * (DK + 4) + KC * DK + 2 * KC * (KC + 4) + DK +
                              DK * SCAN_NC + 2 * KC * SCAN_NC) * sizeof(float);
        if (int rc_ = set_smem(kda_chunk_scan<IO, DK>, (int)smem2)) return rc_;
        const long long nblk = (long long)n_seq * H * (DK / SCAN_NC);
        if (nblk > 0) {
            kda_chunk_scan<IO, DK><<<(unsigned)nblk, 256, smem2, ctx->stream>>>(
                d_table, d_c0, d_c0 + n_seq + 1, (const IO *)v, blocks, state, (IO *)o, H);
            return after_launch(ctx, "kda_chunk_scan");
        }
        (void)L::floats;
        return K3CUDA_OK;
    }
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
