// kda_prefill_tc.cu -- KDA chunkwise prefill on tcgen05 (bf16 operands, fp32 accumulation).
//
// The tensor-core form of kda_prefill.cu's algorithm (same chunk algebra, reference
// src/core/k3_ops.c:908-938 / :186-243), for bf16 q/k/v/o with d_k = d_v = 128. Per chunk
// of C = 64 tokens with G_t = sum_{u<=t} g_u (per key channel):
//
//   Akk[t][s] = beta_t sum_i k_ti k_si e^(G_ti - G_si)   (s < t)
//   Aqk[t][s] =        sum_i q_ti k_si e^(G_ti - G_si)   (s <= t, q pre-scaled)
//   M  = (I + Akk)^-1 diag(beta),  W = M Ktil,  U = M V   (Ktil_t = k_t e^(G_t))
//   Kbar_t = k_t e^(G_C - G_t),    Qtil_t = q_t e^(G_t),   Gamma = e^(G_C)
//
// and the chunk step  X = U - W S,  O = Qtil S + Aqk X,  S' = Gamma S + Kbar^T X  is
// regrouped into its transition form
//
//   S' = Gamma S + P S + Kbar^T U          P  = -Kbar^T W          [d_k x d_k]
//   O  = Q' S + Aqk U                      Q' = Qtil - Aqk W       [C x d_k]
//
// so every product that does not involve S is formed once per (chunk, head) in parallel,
// and the sequential scan over chunks is one batch of MMAs per chunk.
//
//   kda_prep_tc   one CTA per (chunk, head), two CTAs per SM. g, q, k arrive by TMA;
//       G by a per-channel prefix sum; then one vectorised pass (each thread: one token
//       of each 16-token sub-block, eight channels) forms every elementwise operand:
//         A  = [k_t e^(G_t - G_r(t)) ; q_t e^(G_t - G_r(t))]   128 x 128, r(t) = first
//              token of t's sub-block: exponents <= 0
//         B_a[s] = k_s e^(G_r(a) - G_s), s < 16(a+1)            exponent > 0 only inside
//              sub-block a (at most 15 decay steps; a larger one is flagged and that
//              sub-block's columns are recomputed exactly)
//         Ktil, Qtil (in place over k, q), Kbar (to the workspace).
//       Akk and Aqk for row sub-block a come out of one M=128 MMA, A . B_a^T (four
//       "rounds", N = 16, 32, 48, 64). (I + Akk)^-1 by 16x16 blocks in fp32 on the CUDA
//       cores; W = M Ktil, U = M V (M as bf16 hi + lo); P = -Kbar^T W (M=128, N=128,
//       K=64) and Aqk W on tcgen05. Writes P, Kbar, U, Q', Aqk (bf16; Aqk also its
//       bf16 remainder) and Gamma (fp32).
//   kda_scan_tc   one CTA per (sequence, head, 64-column half of d_v). The fp32 state
//       slice lives in TMEM; per chunk the compute warps write its bf16 copy S16 to shared
//       memory and scale the TMEM copy by Gamma (read two chunks ahead from the workspace),
//       then one thread issues
//           S += P . S16 + Kbar^T . U      (M=128, N=64)
//           O  = Q' . S16 + Aqk . U        (M=64,  N=64, double-buffered in TMEM; Aqk as
//                                            bf16 hi + lo)
//       while TMA streams the next chunk's operands (and prefetches later ones into L2).
//
// Operand precision: every tensor-core operand is bf16 and every accumulation fp32; the
// state itself stays fp32 (Gamma is applied in fp32, and only the products with P and Q'
// see its bf16 copy). fp32 I/O takes kda_prefill.cu's fp32 intra-chunk kernel and its
// tensor-core scan over bf16 hi + lo operands (fp32-level products).
#include <vector>

#include "internal.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace k3 {

using namespace sm100;

constexpr int TC_C = 64;    // chunk
constexpr int TC_D = 128;   // d_k = d_v

// Per-(chunk, head) block written by kda_prep_tc, in bytes (row-major bf16 unless noted).
constexpr int WB_P = 0;                 // P = -Kbar^T W  [128 i][128 i']
constexpr int WB_KB = 32768;            // Kbar           [64 t][128 i]
constexpr int WB_U = 49152;             // U              [64 t][128 j]
constexpr int WB_QP = 65536;            // Q'             [64 t][128 i]
constexpr int WB_A = 81920;             // Aqk            [64 t][64 s]
constexpr int WB_AL = 90112;            // Aqk - bf16(Aqk) [64 t][64 s]
constexpr int WB_G = 98304;             // Gamma          [128] fp32
constexpr int WB_BYTES = 98816;         // a multiple of 256

struct TcChunk {
    int seq, t0, len, pad;
};

// fp32 [64][128] G tile, 16-byte units XOR-swizzled within each 128-byte group so that both
// a channel-per-thread pass (fixed t) and a token-per-thread pass (fixed channels) are free
// of bank conflicts
__device__ __forceinline__ int gsw(int t, int i) {
    const int u = i >> 2;
    return t * 128 + (((u & ~7) | ((u ^ t) & 7)) << 2) + (i & 3);
}

// 2^x on the special-function unit (the intra-chunk kernel keeps G in log2 units)
__device__ __forceinline__ float ex2(float x) { return ex2_approx(x); }
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void ld_g8(const float *Gs, int t, int i0, float *v) {
    const float4 a = *reinterpret_cast<const float4 *>(Gs + gsw(t, i0));
    const float4 b = *reinterpret_cast<const float4 *>(Gs + gsw(t, i0 + 4));
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void ld_f8(const float *p, float *v) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0];
    const float4 b = reinterpret_cast<const float4 *>(p)[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

struct PrepMaps {
    CUtensorMap q, k, v, g;         // inputs (loads)
    CUtensorMap p, kb, u, qp, a, al;  // workspace (stores), the scan's maps
};

// Shared memory of kda_prep_tc (bytes from a 1024-aligned base); regions are reused as the
// kernel proceeds. Every swizzled operand starts on a 1024-byte boundary (the hardware
// derives the swizzle from the address bits).
constexpr int PS_Q = 0;                  // q -> Qtil                 [64][128] bf16 (2 k-blocks)
constexpr int PS_K = 16384;              // k -> Ktil -> W            [64][128] bf16
constexpr int PS_R1 = 32768;             // g/G fp32 -> A [128][128] bf16 -> V | Kbar
constexpr int PS_V = PS_R1;              //   V    [64][128] bf16 (MN-major B of U = M V)
constexpr int PS_KBAR = PS_R1 + 16384;   //   Kbar [64][128] bf16 (MN-major A of Kbar^T W)
constexpr int PS_R2 = 65536;             // B_0 | B_1 | B_3, then B_2; then AT, Y, M
constexpr int PS_B0 = PS_R2;             //   16 rows, k-blocks of 2 KB
constexpr int PS_B1 = PS_R2 + 4096;      //   32 rows, k-blocks of 4 KB
constexpr int PS_B3 = PS_R2 + 12288;     //   64 rows, k-blocks of 8 KB
constexpr int PS_B2 = PS_R2;             //   48 rows, k-blocks of 6 KB (second phase)
constexpr int PS_AT = PS_R2;             //   Akk (strictly lower) / T^T (upper) fp32 [64][68]
constexpr int PS_Y = PS_R2 + 17408;      //   block-product scratch, fp32 [32][36]
constexpr int PS_M = PS_R2 + 20480;      //   M bf16 [64][64] (over the dead tail of Y)
constexpr int PS_AQ = 94208;             // Aqk bf16 [64][64] (A of Aqk W)
constexpr int PS_D = 102400;             // D(a,b) = e^(G_r(a) - G_r(b)) fp32 [6][128]
constexpr int PS_EZ = PS_D + 3072;       // e^(G_r(a)) fp32 [4][128]
constexpr int PS_AL = PS_D;              //   then Aqk - bf16(Aqk) bf16 [64][64] (stored out)
constexpr int PS_ML = PS_D;              //   then M - bf16(M) bf16 [64][64]
constexpr int PS_BETA = PS_D + 8192;     // beta [64]
constexpr int PS_BYTES = PS_BETA + 256;
constexpr int PS_SMEM = PS_BYTES + 1024;
constexpr int ATS = 68;                  // AT row stride in floats (16-byte aligned rows)
static_assert(PS_AT + 64 * ATS * 4 <= PS_Y && PS_Y + 32 * 36 * 4 <= PS_AQ &&
                  PS_M + 8192 <= PS_AQ && PS_B3 + 16384 <= PS_AQ,
              "prep shared-memory regions overlap");
static_assert(PS_M % 1024 == 0 && PS_AQ % 1024 == 0 && PS_B2 % 1024 == 0 && PS_B3 % 1024 == 0 &&
                  PS_ML % 1024 == 0 && PS_EZ + 2048 <= PS_BETA,
              "swizzled operands need 1024-byte alignment");

// TMEM column of round a's accumulator (N = 16 (a + 1) columns each)
__device__ __forceinline__ int round_col(int a) { return 8 * a * (a + 1); }
// largest sub-block growth factor 2^x the factored form admits (e^80); beyond it the
// sub-block's columns take the exact path
constexpr float kOverflowLog2 = 80.f * kLog2e;
// index of D(a, b), b < a
__host__ __device__ constexpr int dpair(int a, int b) { return a * (a - 1) / 2 + b; }

__global__ void __launch_bounds__(256, 2)
kda_prep_tc(const __grid_constant__ PrepMaps maps, const TcChunk *__restrict__ chunks,
            const float *__restrict__ gate, const float *__restrict__ beta,
            const __nv_bfloat16 *__restrict__ qg, const __nv_bfloat16 *__restrict__ kg,
            uint8_t *__restrict__ ws, int H, float q_scale, int gate_is_log,
            unsigned *__restrict__ err) {
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar_g, bar_qk, bar_v, bar_mma;
    __shared__ uint32_t tslot;
    __shared__ int flags[4];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const TcChunk cd = chunks[blockIdx.x];
    const int h = blockIdx.y, len = cd.len;
    uint8_t *outb = ws + ((size_t)blockIdx.x * H + h) * WB_BYTES;
    float *Gs = reinterpret_cast<float *>(sm + PS_R1);
    float *Dt = reinterpret_cast<float *>(sm + PS_D);
    float *Ez = reinterpret_cast<float *>(sm + PS_EZ);
    float *sb = reinterpret_cast<float *>(sm + PS_BETA);
    float *AT = reinterpret_cast<float *>(sm + PS_AT);
    float *Y = reinterpret_cast<float *>(sm + PS_Y);

    if (tid == 0) {
        mbar_init(&bar_g, 1);
        mbar_init(&bar_qk, 1);
        mbar_init(&bar_v, 1);
        mbar_init(&bar_mma, 1);
        fence_barrier_init();
        mbar_expect_tx(&bar_g, 32768);
        tma_load_3d(sm + PS_R1, &maps.g, &bar_g, 0, h, cd.t0);
        mbar_expect_tx(&bar_qk, 32768);
        for (int kb = 0; kb < 2; kb++) {
            tma_load_3d(sm + PS_Q + kb * 8192, &maps.q, &bar_qk, kb * 64, h, cd.t0);
            tma_load_3d(sm + PS_K + kb * 8192, &maps.k, &bar_qk, kb * 64, h, cd.t0);
        }
    }
    if (tid < 4) flags[tid] = 0;
    if (tid < TC_C) sb[tid] = tid < len ? beta[(size_t)(cd.t0 + tid) * H + h] : 0.f;
    if (warp == 0) tmem_alloc(&tslot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tslot;
    bool ok = mbar_wait(&bar_g, 0, err, 0x501);

    // ------------------------------------------------------------- G = cumsum(g)
    {
        const int i = tid & 127, half = tid >> 7;
        float gv[32];
#pragma unroll
        for (int r = 0; r < 32; r++) gv[r] = Gs[(32 * half + r) * 128 + i];  // dense, as loaded
        __syncthreads();  // every thread holds its gates: the tile is rewritten swizzled
        // G in log2 units: every use below is 2^(difference of G values)
        if (gate_is_log) {
#pragma unroll
            for (int r = 0; r < 32; r++) gv[r] *= kLog2e;
        } else {
#pragma unroll
            for (int r = 0; r < 32; r++) gv[r] = 32 * half + r < len ? log2f(gv[r]) : 0.f;
        }
        float acc = 0.f;
#pragma unroll
        for (int r = 0; r < 32; r++) {
            acc += 32 * half + r < len ? gv[r] : 0.f;
            gv[r] = acc;
        }
        if (half == 0) {
#pragma unroll
            for (int r = 0; r < 32; r++) Gs[gsw(r, i)] = gv[r];
        }
        __syncthreads();
        if (half == 1) {
            const float base = Gs[gsw(31, i)];
#pragma unroll
            for (int r = 0; r < 32; r++) Gs[gsw(32 + r, i)] = gv[r] + base;
        }
        __syncthreads();
    }
    // per-channel tables: sub-block ratios, decay from the chunk start, Gamma
    if (tid < 128) {
        const int i = tid;
        float gr[4];
#pragma unroll
        for (int a = 0; a < 4; a++) gr[a] = Gs[gsw(16 * a, i)];
#pragma unroll
        for (int a = 1; a < 4; a++)
#pragma unroll
            for (int b = 0; b < a; b++) Dt[dpair(a, b) * 128 + i] = ex2(gr[a] - gr[b]);
#pragma unroll
        for (int a = 0; a < 4; a++) Ez[a * 128 + i] = ex2(gr[a]);
        reinterpret_cast<float *>(outb + WB_G)[i] = ex2(Gs[gsw(63, i)]);
    }
    ok = mbar_wait(&bar_qk, 0, err, 0x502) && ok;
    __syncthreads();

    // -------------------------------------------------- elementwise operands (one pass)
    // thread: channels [8 cc, 8 cc + 8), token j + 16 m of every sub-block m
    // The A rows go over G (same region): this pass leaves them in place of k and q, and a
    // second pass, once every thread has read its G values, moves them into A and scales
    // them by e^(G_r(t)) into Ktil and Qtil.
    const int cc = 2 * warp + (lane >> 4), j = lane & 15, kbk = cc >> 3, ch = cc & 7;
    const int i0 = 8 * cc;
    uint4 b2[3];    // rows of B_2, written once MMA round 2's buffer is free
    uint4 kbar[4];  // Kbar rows, stored once the first region is free
    {
        float gc[8];
        ld_g8(Gs, 63, i0, gc);
        int fl = 0;
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const int t = j + 16 * m;
            float gt[8], ga[8], kv[8], qv[8];
            ld_g8(Gs, t, i0, gt);
            ld_g8(Gs, 16 * m, i0, ga);
            const uint32_t so = (uint32_t)kbk * 8192 + swz(t, ch);
            unpack_bf8(*reinterpret_cast<const uint4 *>(sm + PS_K + so), kv);
            unpack_bf8(*reinterpret_cast<const uint4 *>(sm + PS_Q + so), qv);
            float ak[8], aq[8], bo[8], kb8[8];
            float emax = 0.f;
#pragma unroll
            for (int x = 0; x < 8; x++) {
                const float f = ex2(gt[x] - ga[x]);
                const float e = ga[x] - gt[x];  // >= 0: at most 15 decay steps, in log2 units
                emax = fmaxf(emax, e);
                ak[x] = kv[x] * f;
                aq[x] = qv[x] * (q_scale * f);
                bo[x] = kv[x] * ex2(fminf(e, kOverflowLog2));
                kb8[x] = t < len ? kv[x] * ex2(gc[x] - gt[x]) : 0.f;
            }
            if (emax > kOverflowLog2) fl |= 1 << m;
            st16s(sm + PS_K + so, pack_bf8(ak));
            st16s(sm + PS_Q + so, pack_bf8(aq));
            kbar[m] = pack_bf8(kb8);
            // B_a rows: own sub-block (exponent >= 0), later sub-blocks via D(a, m) <= 1
            if (m == 0) st16s(sm + PS_B0 + kbk * 2048 + swz(t, ch), pack_bf8(bo));
            if (m == 1) st16s(sm + PS_B1 + kbk * 4096 + swz(t, ch), pack_bf8(bo));
            if (m == 2) b2[2] = pack_bf8(bo);
            if (m == 3) st16s(sm + PS_B3 + kbk * 8192 + swz(t, ch), pack_bf8(bo));
#pragma unroll
            for (int a2 = m + 1; a2 < 4; a2++) {
                float dd[8], bv[8];
                ld_f8(Dt + dpair(a2, m) * 128 + i0, dd);
#pragma unroll
                for (int x = 0; x < 8; x++) bv[x] = bo[x] * dd[x];
                if (a2 == 1) st16s(sm + PS_B1 + kbk * 4096 + swz(t, ch), pack_bf8(bv));
                if (a2 == 2) b2[m] = pack_bf8(bv);
                if (a2 == 3) st16s(sm + PS_B3 + kbk * 8192 + swz(t, ch), pack_bf8(bv));
            }
        }
        if (fl) {
#pragma unroll
            for (int m = 0; m < 4; m++)
                if ((fl >> m) & 1) atomicOr(&flags[m], 1);
        }
    }
    __syncthreads();  // G is dead: the A operand goes over it
#pragma unroll
    for (int m = 0; m < 4; m++) {
        const int t = j + 16 * m;
        const uint32_t so = (uint32_t)kbk * 8192 + swz(t, ch);
        const uint4 ak = *reinterpret_cast<const uint4 *>(sm + PS_K + so);
        const uint4 aq = *reinterpret_cast<const uint4 *>(sm + PS_Q + so);
        st16s(sm + PS_R1 + kbk * 16384 + swz(t, ch), ak);
        st16s(sm + PS_R1 + kbk * 16384 + swz(64 + t, ch), aq);
        float ez[8], kt[8], qt[8];
        ld_f8(Ez + m * 128 + i0, ez);
        unpack_bf8(ak, kt);
        unpack_bf8(aq, qt);
#pragma unroll
        for (int x = 0; x < 8; x++) {
            kt[x] *= ez[x];
            qt[x] *= ez[x];
        }
        st16s(sm + PS_K + so, pack_bf8(kt));
        st16s(sm + PS_Q + so, pack_bf8(qt));
    }
    fence_async_shared();
    tc_fence_before();
    ok = __syncthreads_and(ok ? 1 : 0);

    // ------------------------------------------------------------- Akk, Aqk rounds
    // descriptors: one base per operand, the start-address field advanced by offset >> 4
    const uint64_t dsm = sdesc_kmajor(smem_u32(sm));
    auto issue_round = [&](int a, int bbase) {
        const int N = 16 * (a + 1);
        const uint32_t id = idesc_f16(128, N, false, false);
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
            const int kb = ks >> 2;
            mma_bf16_ss(tb + round_col(a), dsm + ((PS_R1 + kb * 16384 + (ks & 3) * 32) >> 4),
                        dsm + ((bbase + kb * N * 128 + (ks & 3) * 32) >> 4), id, ks ? 1u : 0u);
        }
    };
    if (tid == 0 && ok) {
        tc_fence_after();
        issue_round(0, PS_B0);
        issue_round(1, PS_B1);
        issue_round(3, PS_B3);
        mma_commit(&bar_mma);
    }
    if (ok) ok = mbar_wait(&bar_mma, 0, err, 0x503);
#pragma unroll
    for (int m = 0; m < 3; m++) st16s(sm + PS_B2 + kbk * 6144 + swz(j + 16 * m, ch), b2[m]);
    fence_async_shared();
    tc_fence_before();
    ok = __syncthreads_and(ok ? 1 : 0);
    if (tid == 0 && ok) {
        tc_fence_after();
        issue_round(2, PS_B2);
        mma_commit(&bar_mma);
    }
    tc_fence_after();

    // Read-out (M=128: TMEM lane r = row r). Rows 0-63: Akk row t = r; rows 64-127: Aqk row
    // t = r - 64. Warp w reads columns [32 (w >> 2), +32) of its lane quarter; the two
    // sub-blocks of its 32 rows have their own rounds.
    const int q4 = warp & 3, hf = warp >> 2;
    const uint32_t lb = (uint32_t)(32 * q4) << 16;
    auto readout = [&]() {
        const int r = 32 * q4 + lane, t = r & 63;
        const int alo = 2 * (q4 & 1);
        const bool kside = r < 64;
#pragma unroll
        for (int c16 = 0; c16 < 2; c16++) {
            const int s0 = 32 * hf + 16 * c16;
            float vlo[16], vhi[16];
            if (s0 < 16 * (alo + 1)) {
                tmem_ld16(tb + lb + round_col(alo) + s0, vlo);
            } else {
#pragma unroll
                for (int x = 0; x < 16; x++) vlo[x] = 0.f;
            }
            if (s0 < 16 * (alo + 2)) {
                tmem_ld16(tb + lb + round_col(alo + 1) + s0, vhi);
            } else {
#pragma unroll
                for (int x = 0; x < 16; x++) vhi[x] = 0.f;
            }
            tmem_wait_ld();
            float v[16];
#pragma unroll
            for (int x = 0; x < 16; x++) v[x] = lane >= 16 ? vhi[x] : vlo[x];
            if (kside) {
                const float bt = sb[t];
#pragma unroll
                for (int x = 0; x < 16; x++)
                    if (s0 + x < t) AT[t * ATS + s0 + x] = bt * v[x];
            } else {
#pragma unroll
                for (int x = 0; x < 16; x++) v[x] = s0 + x <= t ? v[x] : 0.f;
                const uint4 p0 = pack_bf8(v), p1 = pack_bf8(v + 8);
                st16s(sm + PS_AQ + swz(t, s0 >> 3), p0);
                st16s(sm + PS_AQ + swz(t, (s0 >> 3) + 1), p1);
                float lo[16];
                unpack_bf8(p0, lo);
                unpack_bf8(p1, lo + 8);
#pragma unroll
                for (int x = 0; x < 16; x++) lo[x] = v[x] - lo[x];
                st16s(sm + PS_AL + swz(t, s0 >> 3), pack_bf8(lo));
                st16s(sm + PS_AL + swz(t, (s0 >> 3) + 1), pack_bf8(lo + 8));
            }
        }
    };
    // (Akk lands over the B operands, so nothing is read out before MMA round 2 completes)
    if (ok) ok = mbar_wait(&bar_mma, 1, err, 0x504);
    tc_fence_after();
    if (ok) readout();
    ok = __syncthreads_and(ok ? 1 : 0);

    // Sub-blocks whose 15-step decay overflowed the factored form: every entry of their
    // columns is recomputed exactly (e^(G_t - G_s) per element), from the inputs in global
    // memory and G rebuilt in the (now free) first region.
    if (ok && (flags[0] | flags[1] | flags[2] | flags[3])) {
        {
            const int i = tid & 127, half = tid >> 7;
            float gv[32];
            float acc = 0.f;
#pragma unroll
            for (int r = 0; r < 32; r++) {
                const int t = 32 * half + r;
                float x = 0.f;
                if (t < len) {
                    const float gg = gate[((size_t)(cd.t0 + t) * H + h) * TC_D + i];
                    x = gate_is_log ? gg : logf(gg);
                }
                acc += x;
                gv[r] = acc;
            }
            if (half == 0)
                for (int r = 0; r < 32; r++) Gs[gsw(r, i)] = gv[r];
            __syncthreads();
            if (half == 1) {
                const float base = Gs[gsw(31, i)];
                for (int r = 0; r < 32; r++) Gs[gsw(32 + r, i)] = gv[r] + base;
            }
            __syncthreads();
        }
        for (int b = 0; b < 4; b++) {
            if (!flags[b]) continue;
            for (int e = tid; e < 16 * TC_C; e += 256) {
                const int t = e >> 4, s = 16 * b + (e & 15);
                if (s > t || t >= len) continue;
                const __nv_bfloat16 *kt = kg + ((size_t)(cd.t0 + t) * H + h) * TC_D;
                const __nv_bfloat16 *qt = qg + ((size_t)(cd.t0 + t) * H + h) * TC_D;
                const __nv_bfloat16 *ks = kg + ((size_t)(cd.t0 + s) * H + h) * TC_D;
                float akk = 0.f, aqk = 0.f;
                for (int i = 0; i < TC_D; i++) {
                    const float f = __expf(Gs[gsw(t, i)] - Gs[gsw(s, i)]) * __bfloat162float(ks[i]);
                    akk += __bfloat162float(kt[i]) * f;
                    aqk += __bfloat162float(qt[i]) * q_scale * f;
                }
                if (s < t) AT[t * ATS + s] = sb[t] * akk;
                const __nv_bfloat16 a16 = __float2bfloat16_rn(aqk);
                const uint32_t so = swz(t, s >> 3) + (s & 7) * 2;
                *reinterpret_cast<__nv_bfloat16 *>(sm + PS_AQ + so) = a16;
                *reinterpret_cast<__nv_bfloat16 *>(sm + PS_AL + so) =
                    __float2bfloat16_rn(aqk - __bfloat162float(a16));
            }
        }
        __syncthreads();
    }
    // V into the first region (its generic-proxy uses are complete), Kbar beside it; Aqk and
    // its remainder out to the workspace
    const int chh = blockIdx.x * H + h;  // this block's index in the workspace
    fence_async_shared();
    __syncthreads();
    if (tid == 0 && ok) {
        mbar_expect_tx(&bar_v, 16384);
        for (int kb = 0; kb < 2; kb++)
            tma_load_3d(sm + PS_V + kb * 8192, &maps.v, &bar_v, kb * 64, h, cd.t0);
        tma_store_3d(&maps.a, sm + PS_AQ, 0, 0, chh);
        tma_store_3d(&maps.al, sm + PS_AL, 0, 0, chh);
        bulk_commit();
    }
#pragma unroll
    for (int m = 0; m < 4; m++) st16s(sm + PS_KBAR + kbk * 8192 + swz(j + 16 * m, ch), kbar[m]);
    fence_async_shared();

    // ------------------------------------------- T = (I + Akk)^-1: 16x16 blocks, merged
    // Akk (beta-scaled) sits strictly below the diagonal of AT; T (unit lower triangular)
    // is stored transposed above it: T[x][y] (x > y) at AT[y][x]. Both L rows and T columns
    // are then contiguous in shared memory. Diagonal 16x16 blocks by forward substitution;
    // then T_10 = -T_11 L_10 T_00 merges 16 -> 32 (twice) and 32 -> 64 (once).
    if (warp < 4 && lane < 16) {
        const int o = 16 * warp, c = lane;
        float tc[16];
#pragma unroll
        for (int r = 0; r < 16; r++) tc[r] = r == c ? 1.f : 0.f;
#pragma unroll
        for (int r = 1; r < 16; r++) {
            float lr[16];
#pragma unroll
            for (int q = 0; q < (r + 3) / 4; q++) {
                const float4 l4 = *reinterpret_cast<const float4 *>(AT + (o + r) * ATS + o + 4 * q);
                lr[4 * q] = l4.x, lr[4 * q + 1] = l4.y, lr[4 * q + 2] = l4.z, lr[4 * q + 3] = l4.w;
            }
            float acc = 0.f;
#pragma unroll
            for (int jj = 0; jj < r; jj++) acc += lr[jj] * tc[jj];
            if (r > c) tc[r] = -acc;
        }
#pragma unroll
        for (int r = 1; r < 16; r++)
            if (r > c) AT[(o + c) * ATS + o + r] = tc[r];
    }
    __syncthreads();
    if (tid == 0 && ok) {
        for (int kb = 0; kb < 2; kb++)
            tma_store_3d(&maps.kb, sm + PS_KBAR + kb * 8192, kb * 64, 0, chh);
        bulk_commit();
    }
    {   // 16 -> 32, both halves: Y = L_10 T_00, then T_10 = -T_11 Y. Lane: row r; the
        // two columns c0, c0 + 1 are shared by a half-warp (T loads broadcast).
        const int hb = warp >> 2, r = lane & 15, c0 = 4 * (warp & 3) + 2 * (lane >> 4);
        const int B = 32 * hb;
        float y0 = 0.f, y1 = 0.f;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            if (4 * q + 3 < c0) continue;  // T_00[j][c] = 0 for j < c
            const float4 l4 = *reinterpret_cast<const float4 *>(AT + (B + 16 + r) * ATS + B + 4 * q);
            const float4 a4 = *reinterpret_cast<const float4 *>(AT + (B + c0) * ATS + B + 4 * q);
            const float4 b4 = *reinterpret_cast<const float4 *>(AT + (B + c0 + 1) * ATS + B + 4 * q);
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, av[4] = {a4.x, a4.y, a4.z, a4.w},
                        bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int x = 0; x < 4; x++) {
                const int jj = 4 * q + x;
                y0 += lv[x] * (jj > c0 ? av[x] : (jj == c0 ? 1.f : 0.f));
                y1 += lv[x] * (jj > c0 + 1 ? bv[x] : (jj == c0 + 1 ? 1.f : 0.f));
            }
        }
        *reinterpret_cast<float2 *>(Y + (16 * hb + r) * 36 + c0) = make_float2(y0, y1);
        __syncthreads();
#pragma unroll
        for (int jj = 0; jj < 15; jj++) {
            const float tv = jj < r ? AT[(B + 16 + jj) * ATS + B + 16 + r] : 0.f;
            const float2 yv = *reinterpret_cast<const float2 *>(Y + (16 * hb + jj) * 36 + c0);
            y0 += tv * yv.x;
            y1 += tv * yv.y;
        }
        AT[(B + c0) * ATS + B + 16 + r] = -y0;
        AT[(B + c0 + 1) * ATS + B + 16 + r] = -y1;
    }
    __syncthreads();
    {   // 32 -> 64: Y = L_BA T_AA (rows 32..63, columns 0..31), then T_BA = -T_BB Y.
        // Lane: row r; warp w: columns 4w..4w+3 (warp-uniform: T loads broadcast).
        const int r = lane, c4 = 4 * warp;
        float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < 8; q++) {
            if (q < warp) continue;  // T_AA[j][c] = 0 for j < c
            const float4 l4 = *reinterpret_cast<const float4 *>(AT + (32 + r) * ATS + 4 * q);
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float4 t4 = *reinterpret_cast<const float4 *>(AT + (c4 + u) * ATS + 4 * q);
                float tv[4] = {t4.x, t4.y, t4.z, t4.w};
                if (q == warp) {
#pragma unroll
                    for (int x = 0; x < 4; x++) tv[x] = x > u ? tv[x] : (x == u ? 1.f : 0.f);
                }
#pragma unroll
                for (int x = 0; x < 4; x++) y[u] += lv[x] * tv[x];
            }
        }
        *reinterpret_cast<float4 *>(Y + r * 36 + c4) = make_float4(y[0], y[1], y[2], y[3]);
        __syncthreads();
        // T_BA = -T_BB Y with lane = column c and warp w = rows 4w..4w+3: the triangular bound
        // is warp-uniform and the four T_BB entries of a step are one broadcast float4
        const int c = lane, r0 = 4 * warp;
        float a4[4];
#pragma unroll
        for (int u = 0; u < 4; u++) a4[u] = Y[(r0 + u) * 36 + c];
#pragma unroll
        for (int jj = 0; jj < 31; jj++) {
            if (jj < r0 + 3) {
                const float4 t4 = *reinterpret_cast<const float4 *>(AT + (32 + jj) * ATS + 32 + r0);
                const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
                const float yv = Y[jj * 36 + c];
#pragma unroll
                for (int u = 0; u < 4; u++) a4[u] += (jj < r0 + u ? tv[u] : 0.f) * yv;
            }
        }
        *reinterpret_cast<float4 *>(AT + c * ATS + 32 + r0) =
            make_float4(-a4[0], -a4[1], -a4[2], -a4[3]);
    }
    if (tid == 0) bulk_wait_read<0>();  // the remainder of M goes over the stored-out Aqk
    __syncthreads();
    // M = T diag(beta) as bf16 hi + lo, K-major [t][s]
    for (int u = tid; u < 512; u += 256) {
        const int t = u & 63, c8 = u >> 6;  // a warp: 32 consecutive tokens, one 8-column group
        float mv[8], hi[8];
#pragma unroll
        for (int x = 0; x < 8; x++) {
            const int s = 8 * c8 + x;
            mv[x] = (s < t ? AT[s * ATS + t] : (s == t ? 1.f : 0.f)) * sb[s];
        }
        const uint4 ph = pack_bf8(mv);
        unpack_bf8(ph, hi);
#pragma unroll
        for (int x = 0; x < 8; x++) mv[x] -= hi[x];
        st16s(sm + PS_M + swz(t, c8), ph);
        st16s(sm + PS_ML + swz(t, c8), pack_bf8(mv));
    }
    if (ok) ok = mbar_wait(&bar_v, 0, err, 0x505);
    fence_async_shared();
    tc_fence_before();
    ok = __syncthreads_and(ok ? 1 : 0);

    // ------------------------------------------------------- W = M Ktil, U = M V
    if (tid == 0 && ok) {
        tc_fence_after();
        constexpr uint32_t idw = idesc_f16(64, 128, false, true);
        const uint64_t dmn = sdesc_mnmajor(smem_u32(sm), 8192);
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
            const uint64_t ad = dsm + (((ks < 4 ? PS_M : PS_ML) + (ks & 3) * 32) >> 4);
            mma_bf16_ss(tb, ad, dmn + ((PS_K + (ks & 3) * 2048) >> 4), idw, ks ? 1u : 0u);
            mma_bf16_ss(tb + 128, ad, dmn + ((PS_V + (ks & 3) * 2048) >> 4), idw, ks ? 1u : 0u);
        }
        mma_commit(&bar_mma);
    }
    if (ok) ok = mbar_wait(&bar_mma, 0, err, 0x506);
    tc_fence_after();
    // M=64 accumulators: row 16 q + l in lane l (< 16) of quarter q; warp w reads columns
    // [64 (w >> 2), +64). W goes to shared memory (over Ktil, consumed), U to the workspace.
    if (ok) {
        const int t = 16 * q4 + lane;
#pragma unroll
        for (int c32 = 0; c32 < 2; c32++) {
            float wv[32], uv[32];
            tmem_ld32(tb + lb + 64 * hf + 32 * c32, wv);
            tmem_ld32(tb + lb + 128 + 64 * hf + 32 * c32, uv);
            tmem_wait_ld();
            if (lane < 16) {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    st16s(sm + PS_K + hf * 8192 + swz(t, 4 * c32 + c), pack_bf8(wv + 8 * c));
                    st16s(sm + PS_V + hf * 8192 + swz(t, 4 * c32 + c), pack_bf8(uv + 8 * c));
                }
            }
        }
    }
    fence_async_shared();
    tc_fence_before();
    ok = __syncthreads_and(ok ? 1 : 0);

    // --------------------------------------------- Kbar^T W (M=128) and Aqk W (M=64)
    if (tid == 0 && ok) {
        tc_fence_after();
        for (int kb = 0; kb < 2; kb++) tma_store_3d(&maps.u, sm + PS_V + kb * 8192, kb * 64, 0, chh);
        bulk_commit();
        constexpr uint32_t idp = idesc_f16(128, 128, true, true);
        constexpr uint32_t ida = idesc_f16(64, 128, false, true);
        const uint64_t dmn = sdesc_mnmajor(smem_u32(sm), 8192);
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            const uint64_t bw = dmn + ((PS_K + ks * 2048) >> 4);
            mma_bf16_ss(tb, dmn + ((PS_KBAR + ks * 2048) >> 4), bw, idp, ks ? 1u : 0u);
            mma_bf16_ss(tb + 128, dsm + ((PS_AQ + ks * 32) >> 4), bw, ida, ks ? 1u : 0u);
        }
        mma_commit(&bar_mma);
    }
    if (ok) ok = mbar_wait(&bar_mma, 1, err, 0x507);
    tc_fence_after();
    if (ok) {
        const int i = 32 * q4 + lane;  // row of P
        const int t = 16 * q4 + lane;  // row of Q' (lane < 16)
#pragma unroll
        for (int c32 = 0; c32 < 2; c32++) {
            float pv[32], dv[32];
            tmem_ld32(tb + lb + 64 * hf + 32 * c32, pv);
            tmem_ld32(tb + lb + 128 + 64 * hf + 32 * c32, dv);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 32; x++) pv[x] = -pv[x];
            // P half hf ([128][64]) over the dead AT/M (hf 0) or Kbar (hf 1) tiles
            uint8_t *pb = sm + (hf ? PS_KBAR : PS_R2);
#pragma unroll
            for (int c = 0; c < 4; c++) st16s(pb + swz(i, 4 * c32 + c), pack_bf8(pv + 8 * c));
            if (lane < 16) {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    uint8_t *qa = sm + PS_Q + hf * 8192 + swz(t, 4 * c32 + c);
                    float qt[8];
                    unpack_bf8(*reinterpret_cast<const uint4 *>(qa), qt);
#pragma unroll
                    for (int x = 0; x < 8; x++) qt[x] -= dv[8 * c + x];
                    st16s(qa, pack_bf8(qt));  // Q' over Qtil
                }
            }
        }
    }
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        if (ok) {
            tma_store_3d(&maps.p, sm + PS_R2, 0, 0, chh);
            tma_store_3d(&maps.p, sm + PS_KBAR, 64, 0, chh);
            for (int kb = 0; kb < 2; kb++)
                tma_store_3d(&maps.qp, sm + PS_Q + kb * 8192, kb * 64, 0, chh);
            bulk_commit();
        }
        bulk_wait_read<0>();  // shared memory stays valid until the stores have read it
    }
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tmem_dealloc(tb, 256);
    }
}

// ------------------------------------------------------------------------------ scan
struct ScanMaps {
    CUtensorMap p, kb, u, qp, a, al;
};

// Shared-memory plan of kda_scan_tc for DVT state columns per CTA (the launch uses 64: two
// CTAs per head; 128, one CTA per head, also fits and measured slower). Operand stage (bytes
// from a 1024-aligned base):
template <int DVT>
struct ScanCfg {
    static constexpr int P = 0;                      // P    [128][128]: 2 k-blocks [128][64]
    static constexpr int KB = 32768;                 // Kbar [64][128]:  2 blocks [64 t][64 i]
    static constexpr int QP = 49152;                 // Q'   [64][128]:  2 k-blocks
    static constexpr int U = 65536;                  // U    DVT/64 blocks [64 t][64 j]
    static constexpr int A = U + DVT * 128;          // Aqk  [64][64]
    static constexpr int AL = A + 8192;              // Aqk - bf16(Aqk)
    static constexpr int TX = AL + 8192;             // bytes per stage
    static constexpr int STAGE = (TX + 1023) & ~1023;
    // bf16 copy of the state, [128 i][DVT j] MN-major (64-column atoms of 16 KB); two copies
    // at DVT = 64, one at DVT = 128 (whose next copy then waits for the output products)
    static constexpr int NS16 = DVT == 64 ? 2 : 1;
    static constexpr int S16B = 128 * DVT * 2;
    static constexpr int S16 = 2 * STAGE;
    static constexpr int SMEM = S16 + NS16 * S16B + 1024;
    static constexpr uint32_t TM_COLS = DVT == 64 ? 256 : 512;  // S, O (x2)
};
static_assert(ScanCfg<128>::SMEM <= 232448 && ScanCfg<64>::SMEM <= 232448, "scan shared memory");


// One CTA per (sequence, head, DVT-column slice of d_v). Warps 0-3: thread i owns state row i
// (TMEM lane i) and, for the M=64 output tile, token row 16 w + lane of lanes 0-15; warp 4:
// TMA producer; warp 5: TMEM allocation and MMA issue.
template <int DVT>
__global__ void __launch_bounds__(192, 1)
kda_scan_tc(const __grid_constant__ ScanMaps maps, const TcChunk *__restrict__ chunks,
            const int *__restrict__ seq_chunk0, const int *__restrict__ seq_order,
            const uint8_t *__restrict__ ws,
            float *__restrict__ state, __nv_bfloat16 *__restrict__ o, int H,
            const __grid_constant__ GatherOut go, unsigned *__restrict__ err) {
    using C = ScanCfg<DVT>;
    constexpr int NT = TC_D / DVT;
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t op_full[2], op_empty[2], s_done, o_done[2], s16_ready;
    __shared__ uint32_t tslot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // sequences in descending chunk count: the longest chains are scheduled first
    const int slice = blockIdx.x % NT, h = (blockIdx.x / NT) % H;
    const int n = seq_order[blockIdx.x / (NT * H)];
    const int c0 = seq_chunk0[n], nc = seq_chunk0[n + 1] - c0;
    const int col0 = DVT * slice;
    constexpr uint32_t TM_S = 0, TM_O = DVT;

    if (tid == 0) {
        for (int s = 0; s < 2; s++) {
            mbar_init(&op_full[s], 1);
            mbar_init(&op_empty[s], 1);
            mbar_init(&o_done[s], 1);
        }
        mbar_init(&s_done, 1);
        mbar_init(&s16_ready, 128);
        fence_barrier_init();
    }
    if (warp == 5) tmem_alloc(&tslot, C::TM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tslot;

    if (warp == 4) {
        if (lane == 0) {
            bool ok = true;
            int last[2] = {-1, -1};
            // chunk j + 3 is brought into L2 while chunk j is loaded (two stages cover only
            // one chunk of look-ahead in shared memory)
            auto prefetch = [&](int jj) {
                const int chh = (c0 + jj) * H + h;
                for (int kb = 0; kb < 2; kb++) {
                    tma_prefetch_3d(&maps.p, kb * 64, 0, chh);
                    tma_prefetch_3d(&maps.kb, kb * 64, 0, chh);
                    tma_prefetch_3d(&maps.qp, kb * 64, 0, chh);
                }
                for (int u = 0; u < DVT / 64; u++) tma_prefetch_3d(&maps.u, col0 + 64 * u, 0, chh);
                tma_prefetch_3d(&maps.a, 0, 0, chh);
                tma_prefetch_3d(&maps.al, 0, 0, chh);
            };
            if (nc > 2) prefetch(2);
            for (int j = 0; j < nc && ok; j++) {
                const int st = j & 1, chh = (c0 + j) * H + h;
                if (j + 3 < nc) prefetch(j + 3);
                if (j >= 2 && !(ok = mbar_wait(&op_empty[st], ((j >> 1) - 1) & 1, err, 0x601))) break;
                uint8_t *s = sm + st * C::STAGE;
                mbar_expect_tx(&op_full[st], C::TX);
                for (int kb = 0; kb < 2; kb++) {
                    tma_load_3d(s + C::P + kb * 16384, &maps.p, &op_full[st], kb * 64, 0, chh);
                    tma_load_3d(s + C::KB + kb * 8192, &maps.kb, &op_full[st], kb * 64, 0, chh);
                    tma_load_3d(s + C::QP + kb * 8192, &maps.qp, &op_full[st], kb * 64, 0, chh);
                }
                for (int u = 0; u < DVT / 64; u++)
                    tma_load_3d(s + C::U + u * 8192, &maps.u, &op_full[st], col0 + 64 * u, 0, chh);
                tma_load_3d(s + C::A, &maps.a, &op_full[st], 0, 0, chh);
                tma_load_3d(s + C::AL, &maps.al, &op_full[st], 0, 0, chh);
                last[st] = j;
            }
            // loads still in flight are waited for (bounded) before the CTA may exit
            for (int st = 0; st < 2; st++)
                if (last[st] >= 0) mbar_wait_quiet(&op_full[st], (last[st] >> 1) & 1);
        }
    } else if (warp == 5) {
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_f16(128, DVT, false, true);
            constexpr uint32_t id_k = idesc_f16(128, DVT, true, true);
            constexpr uint32_t id_o = idesc_f16(64, DVT, false, true);
            const uint64_t dk = sdesc_kmajor(smem_u32(sm));
            const uint64_t d8 = sdesc_mnmajor(smem_u32(sm), 8192);     // U, Kbar: 8 KB atoms
            const uint64_t d16 = sdesc_mnmajor(smem_u32(sm), 16384);   // S16: 16 KB atoms
            for (int j = 0; j < nc; j++) {
                const int st = j & 1;
                const int s = st * C::STAGE;
                const int s16 = C::S16 + (C::NS16 == 2 ? (j & 1) * C::S16B : 0);
                if (!mbar_wait(&op_full[st], (j >> 1) & 1, err, 0x602)) break;
                if (!mbar_wait(&s16_ready, j & 1, err, 0x603)) break;
                tc_fence_after();
                // S (already Gamma S) += P . S16 + Kbar^T . U
#pragma unroll
                for (int ks = 0; ks < 8; ks++)
                    mma_bf16_ss(tb + TM_S, dk + ((s + C::P + (ks >> 2) * 16384 + (ks & 3) * 32) >> 4),
                                d16 + ((s16 + ks * 2048) >> 4), id_s, 1u);
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
                    mma_bf16_ss(tb + TM_S, d8 + ((s + C::KB + ks * 2048) >> 4),
                                d8 + ((s + C::U + ks * 2048) >> 4), id_k, 1u);
                mma_commit(&s_done);
                // O = Q' . S16 + Aqk . U
                const uint32_t od = tb + TM_O + DVT * (j & 1);
#pragma unroll
                for (int ks = 0; ks < 8; ks++)
                    mma_bf16_ss(od, dk + ((s + C::QP + (ks >> 2) * 8192 + (ks & 3) * 32) >> 4),
                                d16 + ((s16 + ks * 2048) >> 4), id_o, ks ? 1u : 0u);
#pragma unroll
                for (int ks = 0; ks < 8; ks++)
                    mma_bf16_ss(od, dk + ((s + (ks < 4 ? C::A : C::AL) + (ks & 3) * 32) >> 4),
                                d8 + ((s + C::U + (ks & 3) * 2048) >> 4), id_o, 1u);
                mma_commit(&o_done[j & 1]);
                mma_commit(&op_empty[st]);
            }
        }
    } else if (nc > 0) {
        // ----------------------------------------------------------- compute warps
        const int i = tid;                                // state row / TMEM lane
        const int t = 16 * warp + lane;                   // token row of O (lanes < 16)
        const uint32_t lo = (uint32_t)(32 * warp) << 16;
        float *Sg = state ? state + (((size_t)n * H + h) * TC_D + i) * TC_D + col0 : nullptr;
        float s[64];  // 64 columns of the state row at a time
        // bf16 copy of columns [64 a, +64) of this row into buffer `buf`
        auto write_s16 = [&](int buf, int a) {
            uint8_t *S16 = sm + C::S16 + buf * C::S16B + a * 16384;
#pragma unroll
            for (int c = 0; c < 8; c++) st16s(S16 + swz(i, c), pack_bf8(s + 8 * c));
        };
        auto scale_store = [&](float gam, int a) {
#pragma unroll
            for (int c = 0; c < 64; c += 16) {
                float v[16];
#pragma unroll
                for (int x = 0; x < 16; x++) v[x] = s[c + x] * gam;
                tmem_st16(tb + lo + TM_S + 64 * a + c, v);
            }
        };
        auto load_s = [&](int a) {
#pragma unroll
            for (int c = 0; c < 64; c += 32) tmem_ld32(tb + lo + TM_S + 64 * a + c, s + c);
            tmem_wait_ld();
        };
        // Gamma of chunk jj for this state row, from the workspace (loaded two chunks ahead)
        auto gamma = [&](int jj) {
            return jj < nc ? *reinterpret_cast<const float *>(
                                 ws + ((size_t)(c0 + jj) * H + h) * WB_BYTES + WB_G + 4 * i)
                           : 0.f;
        };
        float gam1 = gamma(1), gam2 = gamma(2);
        // initial state: bf16 copy for the first products, Gamma_0 S_0 into TMEM
        const float gam0 = gamma(0);
#pragma unroll
        for (int a = 0; a < DVT / 64; a++) {
#pragma unroll
            for (int c = 0; c < 64; c += 4) {
                const float4 v = Sg ? *reinterpret_cast<const float4 *>(Sg + 64 * a + c)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                s[c] = v.x, s[c + 1] = v.y, s[c + 2] = v.z, s[c + 3] = v.w;
            }
            write_s16(0, a);
            scale_store(gam0, a);
        }
        tmem_wait_st();
        fence_async_shared();
        tc_fence_before();
        mbar_arrive(&s16_ready);
        bool ok = true;
        TcChunk cd_next = chunks[c0];
        for (int j = 0; j < nc && ok; j++) {
            const TcChunk cd = cd_next;
            if (j + 1 < nc) cd_next = chunks[c0 + j + 1];  // prefetched off the critical path
            if (!(ok = warp_wait_all(&s_done, j & 1, err, 0x605))) break;
            // one copy of S16 (DVT = 128): the output products of chunk j read it too
            if (C::NS16 == 1 && !(ok = warp_wait_all(&o_done[j & 1], (j >> 1) & 1, err, 0x606)))
                break;
            tc_fence_after();
            if (j + 1 < nc) {
#pragma unroll
                for (int a = 0; a < DVT / 64; a++) {
                    load_s(a);
                    write_s16(C::NS16 == 2 ? (j + 1) & 1 : 0, a);
                    scale_store(gam1, a);
                }
                tmem_wait_st();
                gam1 = gam2;
                gam2 = gamma(j + 3);
                fence_async_shared();
                tc_fence_before();
                mbar_arrive(&s16_ready);
            } else if (Sg) {
#pragma unroll
                for (int a = 0; a < DVT / 64; a++) {
                    load_s(a);
#pragma unroll
                    for (int c = 0; c < 64; c += 4)
                        *reinterpret_cast<float4 *>(Sg + 64 * a + c) =
                            make_float4(s[c], s[c + 1], s[c + 2], s[c + 3]);
                }
            }
            // outputs of chunk j (overlapping the next chunk's products)
            if (C::NS16 == 2 && !(ok = warp_wait_all(&o_done[j & 1], (j >> 1) & 1, err, 0x607)))
                break;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < DVT; c += 32) {
                float v[32];
                tmem_ld32(tb + lo + TM_O + DVT * (j & 1) + c, v);
                tmem_wait_ld();
                if (lane < 16 && t < cd.len) {
                    uint4 pk[4];
#pragma unroll
                    for (int q = 0; q < 4; q++) pk[q] = pack_bf8(v + 8 * q);
                    if (go.n == 0) {
                        uint4 *dst = reinterpret_cast<uint4 *>(
                            o + ((size_t)(cd.t0 + t) * H + h) * TC_D + col0 + c);
#pragma unroll
                        for (int q = 0; q < 4; q++) dst[q] = pk[q];
                    } else {
                        // the row goes straight into every rank's full output (peer memory
                        // over NVLink), at this rank's heads of the [T][H_total][dv] layout
                        const size_t off =
                            ((size_t)(cd.t0 + t) * go.H_total + go.head0 + h) * TC_D + col0 + c;
                        for (int r = 0; r < go.n; r++) {
                            uint4 *dst = reinterpret_cast<uint4 *>(go.ptr[r] + off);
#pragma unroll
                            for (int q = 0; q < 4; q++) dst[q] = pk[q];
                        }
                    }
                }
            }
            tc_fence_before();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tmem_dealloc(tb, C::TM_COLS);
    }
}

// -------------------------------------------------------------------------- host side
size_t prefill_tc_block_bytes() { return WB_BYTES; }

// Launch both phases. `blocks` has room for nc * H blocks of WB_BYTES; d_table / d_c0 are
// the device copies of the chunk table and of the per-sequence first-chunk index [n_seq + 1],
// followed by the sequences in descending chunk count [n_seq].
int run_prefill_tc(k3cuda_ctx *ctx, float *state, void *o, const void *q, const void *k,
                   const void *v, const float *gate, const float *beta, int total_tokens,
                   int n_seq, int H, float q_scale, int gate_is_log, long long nc,
                   const void *d_table, const int *d_c0, void *blocks, const GatherOut *go) {
    const GatherOut gout = go ? *go : GatherOut{};
    const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const CUtensorMapDataType F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    PrepMaps pm;
    const uint64_t rs = (uint64_t)H * TC_D * 2;  // bytes per token row of q/k/v
    int rc = make_tmap_3d(&pm.q, q, BF, 2, TC_D, H, total_tokens, TC_D * 2, rs, 64, 1, 64);
    if (!rc) rc = make_tmap_3d(&pm.k, k, BF, 2, TC_D, H, total_tokens, TC_D * 2, rs, 64, 1, 64);
    if (!rc) rc = make_tmap_3d(&pm.v, v, BF, 2, TC_D, H, total_tokens, TC_D * 2, rs, 64, 1, 64);
    if (!rc)
        rc = make_tmap_3d(&pm.g, gate, F32, 4, TC_D, H, total_tokens, TC_D * 4, 2 * rs, 128, 1,
                          64);
    // workspace maps: stores of the intra-chunk kernel, loads of the scan
    const uint64_t nch = (uint64_t)nc * H;
    uint8_t *b = (uint8_t *)blocks;
    if (!rc) rc = make_tmap_3d(&pm.p, b + WB_P, BF, 2, 128, 128, nch, 256, WB_BYTES, 64, 128, 1);
    if (!rc) rc = make_tmap_3d(&pm.kb, b + WB_KB, BF, 2, 128, 64, nch, 256, WB_BYTES, 64, 64, 1);
    if (!rc) rc = make_tmap_3d(&pm.u, b + WB_U, BF, 2, 128, 64, nch, 256, WB_BYTES, 64, 64, 1);
    if (!rc) rc = make_tmap_3d(&pm.qp, b + WB_QP, BF, 2, 128, 64, nch, 256, WB_BYTES, 64, 64, 1);
    if (!rc) rc = make_tmap_3d(&pm.a, b + WB_A, BF, 2, 64, 64, nch, 128, WB_BYTES, 64, 64, 1);
    if (!rc) rc = make_tmap_3d(&pm.al, b + WB_AL, BF, 2, 64, 64, nch, 128, WB_BYTES, 64, 64, 1);
    if (rc) return rc;
    if (int rc_ = set_smem(kda_prep_tc, PS_SMEM)) return rc_;
    kda_prep_tc<<<dim3((unsigned)nc, (unsigned)H), 256, PS_SMEM, ctx->stream>>>(
        pm, (const TcChunk *)d_table, gate, beta, (const __nv_bfloat16 *)q,
        (const __nv_bfloat16 *)k, (uint8_t *)blocks, H, q_scale, gate_is_log, ctx->err_word);
    rc = after_launch(ctx, "kda_prep_tc");
    if (rc) return rc;

    ScanMaps sm{pm.p, pm.kb, pm.u, pm.qp, pm.a, pm.al};
    // Two CTAs per head (64 state columns each): every chunk's chain is half as long as with
    // whole 128-column rows, which also pack the GPU more finely when there are many
    // (sequence, head) pairs (config 3: 6.05 ms with whole rows, 5.98 ms with halves)
    using C = ScanCfg<64>;
    if (int rc_ = set_smem(kda_scan_tc<64>, C::SMEM)) return rc_;
    kda_scan_tc<64><<<(unsigned)((long long)n_seq * H * 2), 192, C::SMEM, ctx->stream>>>(
        sm, (const TcChunk *)d_table, d_c0, d_c0 + n_seq + 1, b, state, (__nv_bfloat16 *)o, H,
        gout, ctx->err_word);
    return after_launch(ctx, "kda_scan_tc");
}

}  // namespace k3
