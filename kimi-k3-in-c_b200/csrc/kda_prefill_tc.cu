// kda_prefill_tc.cu -- KDA chunkwise prefill on tcgen05 (bf16 operands, fp32 accumulation).
//
// The tensor-core form of kda_prefill.cu's algorithm (same chunk algebra, reference
// src/core/k3_ops.c:908-938 / :186-243), for bf16 q/k/v/o with d_k = d_v = 128:
//
//   kda_prep_tc   one CTA per (chunk, head), every chunk in parallel:
//       G = cumsum(g) per key channel; within-sub-block factors F = e^(G_t - G_r),
//       Finv = e^(G_r - G_t) (r = first token of t's 16-token sub-block) and per-channel
//       sub-block ratios D(a,b) = e^(G_r(a) - G_r(b)) -- every exponent <= 0 except Finv's,
//       which spans at most 15 decay steps (a larger one marks its sub-block for the exact
//       path below).
//       Akk, Aqk by column sub-block b: A[:, b] = (k F D(a,b)) . (k Finv)_b^T on tcgen05
//       (M=64 tokens, N=16, K=128 channels), four rounds.
//       (I + diag(beta) Akk)^-1 by 16x16 blocks in fp32 (forward substitution on the four
//       diagonal blocks, then the off-diagonal blocks by block products).
//       W = M Ktil and U = M V on tcgen05 (M = T diag(beta), Ktil = k e^(G_t): the decay
//       from the chunk start through token t).
//       Writes W, U, Qtil = q e^(G_t), Kbar^T = (k e^(G_C - G_t))^T, Aqk (bf16) and
//       Gamma = e^(G_C) (fp32) per (chunk, head).
//   kda_scan_tc   one CTA per (sequence, head, slice of d_v): the fp32 state slice lives
//       in TMEM for the whole sequence; per chunk
//           X = U - W S16          (tcgen05, S16 = bf16 copy of S in shared memory)
//           O = Qtil S16 + Aqk X   (tcgen05)
//           S = Gamma S + Kbar^T X (tcgen05, accumulating into the fp32 state in TMEM)
//
// Operand precision: every tensor-core operand is bf16 and every accumulation fp32. On the
// synthetic distributions of the workloads this holds the outputs and the final state to
// about 2.5e-3 relative Frobenius error of the fp32 recurrence (inside the 5e-3 bar for
// bf16 inputs); fp32 I/O keeps the CUDA-core path of kda_prefill.cu, which is exact to fp32
// rounding.
#include <vector>

#include "internal.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace k3 {

using namespace sm100;

constexpr int TC_C = 64;    // chunk
constexpr int TC_D = 128;   // d_k = d_v

// Per-(chunk, head) block written by kda_prep_tc, in bytes.
constexpr int PB_W = 0;                 // W    [64][128] bf16
constexpr int PB_U = PB_W + 16384;      // U    [64][128] bf16
constexpr int PB_Q = PB_U + 16384;      // Qtil [64][128] bf16
constexpr int PB_KB = PB_Q + 16384;     // Kbar^T [128][64] bf16
constexpr int PB_A = PB_KB + 16384;     // Aqk  [64][64] bf16
constexpr int PB_G = PB_A + 8192;       // Gamma [128] fp32
constexpr int PB_BYTES = PB_G + 512;    // 74240 (a multiple of 256)

struct TcChunk {
    int seq, t0, len, pad;
};

// byte offset of element (r, c), c < 64, inside a [rows x 64 bf16] 128-byte-swizzled block
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t)(r * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + (c & 7) * 2);
}

__device__ __forceinline__ float ldbf(const uint8_t *base, uint32_t off) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(base + off));
}
__device__ __forceinline__ void stbf(uint8_t *base, uint32_t off, float x) {
    *reinterpret_cast<__nv_bfloat16 *>(base + off) = __float2bfloat16_rn(x);
}

struct PrepMaps {
    CUtensorMap q, k, v;
};

// shared memory of kda_prep_tc (bytes from a 1024-aligned base). The tensor-core operands
// come first: a 128-byte-swizzled operand must start on a 1024-byte boundary, because the
// hardware derives the swizzle from the address bits.
constexpr int PS_Q = 0;                       // q tile  2 x [64 x 64] bf16 SW128
constexpr int PS_K = PS_Q + 16384;            // k tile
constexpr int PS_V = PS_K + 16384;            // v tile (MN-major B of U = M V)
constexpr int PS_R = PS_V + 16384;            // R 16K, Rq 16K, Kh 4K; later M 8K, Ktil 16K
constexpr int PS_F = PS_R + 36864;            // F    fp32 [64][129] (33 KB padded)
constexpr int PS_FI = PS_F + 33792;           // Finv fp32 [64][129]
constexpr int PS_G = PS_FI + 33792;           // G fp32 [64][128]; later T [64][65] + Y
constexpr int PS_A = PS_G + 32768;            // Akk fp32 [64][65]
constexpr int PS_D = PS_A + 64 * 65 * 4;      // D(a,b) fp32 [4][4][128]
constexpr int PS_EC = PS_D + 8192;            // e^(G_C - G_r(a)) fp32 [4][128]
constexpr int PS_EZ = PS_EC + 2048;           // e^(G_r(a)) fp32 [4][128]
constexpr int PS_GC = PS_EZ + 2048;           // Gamma fp32 [128]
constexpr int PS_B = PS_GC + 512;             // beta fp32 [64]
constexpr int PS_BYTES = PS_B + 256;
constexpr int PS_SMEM = PS_BYTES + 1024;
static_assert(PS_K % 1024 == 0 && PS_V % 1024 == 0 && PS_R % 1024 == 0,
              "swizzled operands need 1024-byte alignment");
static_assert(64 * 129 * 4 <= 33792, "F padding");

__global__ void __launch_bounds__(256, 1)
kda_prep_tc(const __grid_constant__ PrepMaps maps, const TcChunk *__restrict__ chunks,
            const float *__restrict__ gate, const float *__restrict__ beta,
            uint8_t *__restrict__ ws, int H, float q_scale, int gate_is_log,
            unsigned *__restrict__ err) {
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar_ld, bar_mma;
    __shared__ uint32_t tslot;
    __shared__ int flags[4];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const TcChunk cd = chunks[blockIdx.x];
    const int h = blockIdx.y;
    uint8_t *outb = ws + ((size_t)blockIdx.x * H + h) * PB_BYTES;
    float *F = reinterpret_cast<float *>(sm + PS_F);
    float *Fi = reinterpret_cast<float *>(sm + PS_FI);
    float *G = reinterpret_cast<float *>(sm + PS_G);
    float *A = reinterpret_cast<float *>(sm + PS_A);
    float *Dab = reinterpret_cast<float *>(sm + PS_D);
    float *Ec = reinterpret_cast<float *>(sm + PS_EC);
    float *Ez = reinterpret_cast<float *>(sm + PS_EZ);
    float *Gc = reinterpret_cast<float *>(sm + PS_GC);
    float *sb = reinterpret_cast<float *>(sm + PS_B);
    uint8_t *sQ = sm + PS_Q, *sK = sm + PS_K, *sV = sm + PS_V;

    if (tid == 0) {
        mbar_init(&bar_ld, 1);
        mbar_init(&bar_mma, 1);
        fence_barrier_init();
        mbar_expect_tx(&bar_ld, 3 * 16384);
        for (int kb = 0; kb < 2; kb++) {
            tma_load_3d(sQ + kb * 8192, &maps.q, &bar_ld, kb * 64, h, cd.t0);
            tma_load_3d(sK + kb * 8192, &maps.k, &bar_ld, kb * 64, h, cd.t0);
            tma_load_3d(sV + kb * 8192, &maps.v, &bar_ld, kb * 64, h, cd.t0);
        }
    }
    if (tid < 4) flags[tid] = 0;
    if (warp == 1) tmem_alloc(&tslot, 256);
    // G = cumsum(g): thread (i, half) sums rows [32 half, 32 half + 32) of channel i
    {
        const int i = tid & 127, half = tid >> 7;
        float gv[32];
#pragma unroll
        for (int r = 0; r < 32; r++) {  // all 32 loads in flight before the first add
            const int t = half * 32 + r;
            gv[r] = t < cd.len ? gate[((size_t)(cd.t0 + t) * H + h) * TC_D + i] : 1.f;
        }
        float acc = 0.f;
#pragma unroll
        for (int r = 0; r < 32; r++) {
            const int t = half * 32 + r;
            float x = 0.f;
            if (t < cd.len) x = gate_is_log ? gv[r] : logf(gv[r]);
            acc += x;
            G[t * 128 + i] = acc;
        }
        if (tid < TC_C) sb[tid] = tid < cd.len ? beta[(size_t)(cd.t0 + tid) * H + h] : 0.f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tslot;
    if (tid >= 128) {
        const int i = tid & 127;
        const float base = G[31 * 128 + i];
        for (int t = 32; t < 64; t++) G[t * 128 + i] += base;
    }
    __syncthreads();
    // factors
    for (int e = tid; e < TC_C * 128; e += 256) {
        const int t = e >> 7, i = e & 127, r = t & ~15;
        const float g = G[e], gr = G[r * 128 + i];
        F[t * 129 + i] = __expf(g - gr);
        const float ex = gr - g;
        if (ex > 80.f) atomicOr(&flags[t >> 4], 1);
        Fi[t * 129 + i] = __expf(fminf(ex, 80.f));
    }
    if (tid < 128) {
        const int i = tid;
        for (int a = 0; a < 4; a++) {
            for (int b = 0; b < a; b++)
                Dab[(a * 4 + b) * 128 + i] = __expf(G[16 * a * 128 + i] - G[16 * b * 128 + i]);
            Dab[(a * 4 + a) * 128 + i] = 1.f;
            Ec[a * 128 + i] = __expf(G[63 * 128 + i] - G[16 * a * 128 + i]);
            Ez[a * 128 + i] = __expf(G[16 * a * 128 + i]);  // decay from the chunk start
        }
        Gc[i] = __expf(G[63 * 128 + i]);
    }
    bool ok = true;
    if (tid == 0) ok = mbar_wait(&bar_ld, 0, err, 0x501);
    __syncthreads();
    ok = __syncthreads_and(ok ? 1 : 0) && !*(volatile unsigned *)err;
    // Qtil = q e^(G_t - G_0), Kbar^T = (k e^(G_C - G_t))^T and Gamma = e^(G_C) to the
    // workspace (G is still live here for sub-blocks flagged by the overflow guard)
    for (int e = tid; e < TC_C * 128; e += 256) {
        const int t = e >> 7, i = e & 127;
        float v = 0.f;
        if (t < cd.len)
            v = ldbf(sQ, (i >> 6) * 8192 + sw128(t, i & 63)) * q_scale * F[t * 129 + i] *
                Ez[(t >> 4) * 128 + i];
        stbf(outb + PB_Q, (uint32_t)(t * 128 + i) * 2, v);
    }
    for (int e = tid; e < TC_C * 128; e += 256) {
        const int t = e >> 7, i = e & 127;
        float v = 0.f;
        if (t < cd.len) {
            const float kv = ldbf(sK, (i >> 6) * 8192 + sw128(t, i & 63));
            v = flags[t >> 4] ? kv * __expf(G[63 * 128 + i] - G[t * 128 + i])
                              : kv * Fi[t * 129 + i] * Ec[(t >> 4) * 128 + i];
        }
        stbf(outb + PB_KB, (uint32_t)(i * 64 + t) * 2, v);
    }
    if (tid < 128) reinterpret_cast<float *>(outb + PB_G)[tid] = Gc[tid];

    // ---------------------------------------------------------------- Akk, Aqk
    uint8_t *sR = sm + PS_R, *sRq = sR + 16384, *sKh = sR + 32768;
    constexpr uint32_t id_a = idesc_f16(64, 16, false, false);
    for (int b = 0; b < 4 && ok; b++) {
        for (int e = tid; e < TC_C * 128; e += 256) {
            const int t = e >> 7, i = e & 127, a = t >> 4;
            float rk = 0.f, rq = 0.f;
            if (a >= b && t < cd.len) {
                const float f = F[t * 129 + i] * Dab[(a * 4 + b) * 128 + i];
                const uint32_t off = (i >> 6) * 8192 + sw128(t, i & 63);
                rk = ldbf(sK, off) * f;
                rq = ldbf(sQ, off) * q_scale * f;
            }
            const uint32_t o = (i >> 6) * 8192 + sw128(t, i & 63);
            stbf(sR, o, rk);
            stbf(sRq, o, rq);
        }
        for (int e = tid; e < 16 * 128; e += 256) {
            const int s = e >> 7, i = e & 127, t = 16 * b + s;
            const float v = t < cd.len ? ldbf(sK, (i >> 6) * 8192 + sw128(t, i & 63)) * Fi[t * 129 + i]
                                       : 0.f;
            stbf(sKh, (i >> 6) * 2048 + sw128(s, i & 63), v);
        }
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            for (int kb = 0; kb < 2; kb++)
#pragma unroll
                for (int ks = 0; ks < 4; ks++) {
                    const uint64_t bd = sdesc_kmajor(smem_u32(sKh + kb * 2048 + ks * 32));
                    const uint32_t acc = (kb | ks) ? 1u : 0u;
                    mma_bf16_ss(tb + 16 * b, sdesc_kmajor(smem_u32(sR + kb * 8192 + ks * 32)), bd,
                                id_a, acc);
                    mma_bf16_ss(tb + 64 + 16 * b, sdesc_kmajor(smem_u32(sRq + kb * 8192 + ks * 32)),
                                bd, id_a, acc);
                }
            mma_commit(&bar_mma);
        }
        __syncwarp();
        ok = mbar_wait(&bar_mma, b & 1, err, 0x502);
        ok = __syncthreads_and(ok ? 1 : 0);
        tc_fence_after();
    }
    // read Akk (beta-scaled, strictly lower) to shared memory, Aqk (lower) to the workspace.
    // M=64 accumulator: row 16 w + l sits in lane l (< 16) of warp w's TMEM quarter.
    if (ok && warp < 4) {
        const int t = 16 * warp + lane;
        for (int c = 0; c < 64; c += 16) {
            float vk[16], vq[16];
            tmem_ld16(tb + ((uint32_t)(32 * warp) << 16) + c, vk);
            tmem_ld16(tb + ((uint32_t)(32 * warp) << 16) + 64 + c, vq);
            tmem_wait_ld();
            if (lane < 16) {
                uint32_t pk[8];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int s = c + j;
                    A[t * 65 + s] = s < t ? sb[t] * vk[j] : 0.f;
                    vq[j] = s <= t ? vq[j] : 0.f;
                }
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const __nv_bfloat162 p = __floats2bfloat162_rn(vq[2 * j], vq[2 * j + 1]);
                    pk[j] = *reinterpret_cast<const uint32_t *>(&p);
                }
                uint4 *dst = reinterpret_cast<uint4 *>(outb + PB_A + (t * 64 + c) * 2);
                dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    // column sub-blocks b whose 15-step decay overflowed the factored form (their Finv was
    // clamped): every entry with s in b recomputed exactly, e^(G_t - G_s) per element
    for (int b = 0; b < 4 && ok; b++) {
        if (!flags[b]) continue;
        for (int e = tid; e < 16 * TC_C; e += 256) {
            const int t = e >> 4, s = 16 * b + (e & 15);
            if (s > t || t >= cd.len) continue;
            float akk = 0.f, aqk = 0.f;
            for (int i = 0; i < 128; i++) {
                const uint32_t ot = (i >> 6) * 8192 + sw128(t, i & 63);
                const uint32_t os = (i >> 6) * 8192 + sw128(s, i & 63);
                const float f = __expf(G[t * 128 + i] - G[s * 128 + i]) * ldbf(sK, os);
                akk += ldbf(sK, ot) * f;
                aqk += ldbf(sQ, ot) * q_scale * f;
            }
            A[t * 65 + s] = s < t ? sb[t] * akk : 0.f;
            stbf(outb + PB_A, (uint32_t)(t * 64 + s) * 2, aqk);
        }
    }
    __syncthreads();

    // ------------------------------------------------- T = (I + Akk)^-1, M = T diag(beta)
    float *T = G;                 // [64][65], G is dead from here
    float *Y = G + 64 * 65;       // [3][16][17] scratch
    if (warp < 4 && lane < 16) {
        // diagonal block w, column c = lane: forward substitution, columns independent
        const int o = 16 * warp, c = lane;
        for (int r = 0; r < 16; r++) {
            float v = r == c ? 1.f : 0.f;
            if (r > c) {
                float acc = 0.f;
                for (int j = c; j < r; j++) acc += A[(o + r) * 65 + o + j] * T[(o + j) * 65 + o + c];
                v = -acc;
            }
            T[(o + r) * 65 + o + c] = v;
        }
    }
    __syncthreads();
    for (int d = 1; d < 4; d++) {
        const int nb = 4 - d;  // blocks (a, a-d), a = d..3
        for (int e = tid; e < nb * 256; e += 256) {
            const int a = d + e / 256, b = a - d, r = (e >> 4) & 15, c = e & 15;
            float acc = 0.f;
            for (int m = b; m < a; m++)
                for (int j = 0; j < 16; j++)
                    acc += A[(16 * a + r) * 65 + 16 * m + j] * T[(16 * m + j) * 65 + 16 * b + c];
            Y[(a - d) * 272 + r * 17 + c] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nb * 256; e += 256) {
            const int a = d + e / 256, b = a - d, r = (e >> 4) & 15, c = e & 15;
            float acc = 0.f;
            for (int j = 0; j <= r; j++)
                acc += T[(16 * a + r) * 65 + 16 * a + j] * Y[(a - d) * 272 + j * 17 + c];
            T[(16 * a + r) * 65 + 16 * b + c] = -acc;
        }
        __syncthreads();
    }
    // M (bf16, K-major [t][s]) and Ktil (bf16, MN-major [t][i]) into the freed R region
    uint8_t *sM = sm + PS_R, *sKt = sm + PS_R + 8192;
    for (int e = tid; e < TC_C * TC_C; e += 256) {
        const int t = e >> 6, s = e & 63;
        stbf(sM, sw128(t, s), s <= t ? T[t * 65 + s] * sb[s] : 0.f);
    }
    for (int e = tid; e < TC_C * 128; e += 256) {
        const int t = e >> 7, i = e & 127;
        const uint32_t off = (i >> 6) * 8192 + sw128(t, i & 63);
        float v = 0.f;
        if (t < cd.len) v = ldbf(sK, off) * F[t * 129 + i] * Ez[(t >> 4) * 128 + i];
        stbf(sKt, off, v);
    }
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && ok) {
        tc_fence_after();
        constexpr uint32_t id_w = idesc_f16(64, 128, false, true);
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            const uint64_t ad = sdesc_kmajor(smem_u32(sM + ks * 32));
            mma_bf16_ss(tb, ad, sdesc_mnmajor(smem_u32(sKt + ks * 2048), 8192), id_w, ks ? 1u : 0u);
            mma_bf16_ss(tb + 128, ad, sdesc_mnmajor(smem_u32(sV + ks * 2048), 8192), id_w,
                        ks ? 1u : 0u);
        }
        mma_commit(&bar_mma);
    }
    __syncwarp();
    if (ok) ok = mbar_wait(&bar_mma, 0, err, 0x503);  // 5th commit: phase 0 of round parity
    ok = __syncthreads_and(ok ? 1 : 0);
    tc_fence_after();
    if (ok && warp < 4) {
        const int t = 16 * warp + lane;
        for (int which = 0; which < 2; which++)
            for (int c = 0; c < 128; c += 16) {
                float v[16];
                tmem_ld16(tb + ((uint32_t)(32 * warp) << 16) + which * 128 + c, v);
                tmem_wait_ld();
                if (lane < 16) {
                    uint32_t pk[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                        pk[j] = *reinterpret_cast<const uint32_t *>(&p);
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(outb + (which ? PB_U : PB_W) +
                                                           (t * 128 + c) * 2);
                    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
            }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tb, 256);
    }
}

}  // namespace k3

namespace k3 {

struct ScanMaps {
    CUtensorMap w, q, kb, a, u, g;
};

__device__ __forceinline__ bool warp_wait_all(uint64_t *bar, uint32_t parity, unsigned *err,
                                              unsigned code) {
    const bool ok = mbar_wait(bar, parity, err, code);
    return __all_sync(0xffffffffu, ok);
}

// One CTA per (sequence, head, DVT-column slice of d_v). Warps 0-3: one thread per TMEM
// lane (state row i; for the M=64 products, token row 16 w + lane of lanes 0-15); warp 4:
// TMA producer; warp 5: TMEM allocation and MMA issue.
template <int DVT>
__global__ void __launch_bounds__(192, 1)
kda_scan_tc(const __grid_constant__ ScanMaps maps, const TcChunk *__restrict__ chunks,
            const int *__restrict__ seq_chunk0, const uint8_t *__restrict__ ws,
            float *__restrict__ state, __nv_bfloat16 *__restrict__ o, int H,
            unsigned *__restrict__ err) {
    // operand stage: W, Qtil, Kbar^T, Aqk, U slice, Gamma (padded to 1 KB)
    constexpr int OFF_GAM = 57344 + 128 * DVT;
    constexpr int STAGE_TX = OFF_GAM + 512;
    constexpr int SB = (STAGE_TX + 1023) & ~1023;
    static_assert(SB % 1024 == 0 && (DVT * 256) % 1024 == 0, "1024-byte aligned operands");
    constexpr int OFF_S16 = 2 * SB;               // bf16 S^T [DVT][128] (2 K-blocks)
    constexpr int OFF_XT = OFF_S16 + DVT * 256;   // bf16 X^T [DVT][64]
    constexpr int TM_S = 0, TM_X = DVT, TM_O = 2 * DVT;
    constexpr uint32_t TM_COLS = DVT <= 32 ? 128 : 512;
    constexpr int NT = TC_D / DVT;
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t op_full[2], op_empty[2], x_full, xt_ready, done, s16_ready;
    __shared__ uint32_t tslot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x % NT, h = (blockIdx.x / NT) % H, n = blockIdx.x / (NT * H);
    const int c0 = seq_chunk0[n], nc = seq_chunk0[n + 1] - c0;
    const int col0 = tile * DVT;
    uint8_t *S16 = sm + OFF_S16, *XT = sm + OFF_XT;

    if (tid == 0) {
        for (int s = 0; s < 2; s++) {
            mbar_init(&op_full[s], 1);
            mbar_init(&op_empty[s], 1);
        }
        mbar_init(&x_full, 1);
        mbar_init(&xt_ready, 128);
        mbar_init(&done, 1);
        mbar_init(&s16_ready, 128);
        fence_barrier_init();
    }
    if (warp == 5) tmem_alloc(&tslot, TM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tslot;

    if (warp == 4) {
        if (lane == 0) {
            bool ok = true;
            int last[2] = {-1, -1};
            for (int j = 0; j < nc && ok; j++) {
                const int st = j & 1, ch = (c0 + j) * H + h;
                if (j >= 2 && !(ok = mbar_wait(&op_empty[st], ((j >> 1) - 1) & 1, err, 0x601))) break;
                uint8_t *s = sm + st * SB;
                mbar_expect_tx(&op_full[st], STAGE_TX);
                for (int kb = 0; kb < 2; kb++) {
                    tma_load_3d(s + kb * 8192, &maps.w, &op_full[st], kb * 64, 0, ch);
                    tma_load_3d(s + 16384 + kb * 8192, &maps.q, &op_full[st], kb * 64, 0, ch);
                }
                tma_load_3d(s + 32768, &maps.kb, &op_full[st], 0, 0, ch);
                tma_load_3d(s + 49152, &maps.a, &op_full[st], 0, 0, ch);
                for (int u = 0; u < (DVT + 63) / 64; u++)
                    tma_load_3d(s + 57344 + u * 8192, &maps.u, &op_full[st], col0 + u * 64, 0, ch);
                tma_load_2d(s + OFF_GAM, &maps.g, &op_full[st], 0, ch);
                last[st] = j;
            }
            // loads still in flight are waited for (bounded) before the CTA may exit
            for (int st = 0; st < 2; st++)
                if (last[st] >= 0) mbar_wait_quiet(&op_full[st], (last[st] >> 1) & 1);
        }
    } else if (warp == 5) {
        if (lane == 0) {
            constexpr uint32_t id64 = idesc_f16(64, DVT, false, false);
            constexpr uint32_t id128 = idesc_f16(128, DVT, false, false);
            for (int j = 0; j < nc; j++) {
                const int st = j & 1;
                const uint8_t *s = sm + st * SB;
                if (!mbar_wait(&op_full[st], (j >> 1) & 1, err, 0x602)) break;
                if (!mbar_wait(&s16_ready, j & 1, err, 0x603)) break;
                tc_fence_after();
                // X_acc = W . S16 ; O = Qtil . S16
                for (int kb = 0; kb < 2; kb++)
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        mma_bf16_ss(tb + TM_X, sdesc_kmajor(smem_u32(s + kb * 8192 + ks * 32)),
                                    sdesc_kmajor(smem_u32(S16 + kb * DVT * 128 + ks * 32)), id64,
                                    (kb | ks) ? 1u : 0u);
                mma_commit(&x_full);
                for (int kb = 0; kb < 2; kb++)
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        mma_bf16_ss(tb + TM_O, sdesc_kmajor(smem_u32(s + 16384 + kb * 8192 + ks * 32)),
                                    sdesc_kmajor(smem_u32(S16 + kb * DVT * 128 + ks * 32)), id64,
                                    (kb | ks) ? 1u : 0u);
                if (!mbar_wait(&xt_ready, j & 1, err, 0x604)) break;
                tc_fence_after();
                // S += Kbar^T . X ; O += Aqk . X
#pragma unroll
                for (int ks = 0; ks < 4; ks++) {
                    const uint64_t bx = sdesc_kmajor(smem_u32(XT + ks * 32));
                    mma_bf16_ss(tb + TM_S, sdesc_kmajor(smem_u32(s + 32768 + ks * 32)), bx, id128, 1u);
                    mma_bf16_ss(tb + TM_O, sdesc_kmajor(smem_u32(s + 49152 + ks * 32)), bx, id64, 1u);
                }
                mma_commit(&done);
                mma_commit(&op_empty[st]);
            }
        }
    } else {
        // ----------------------------------------------------------- compute warps
        const int i = 32 * warp + lane;                 // state row / TMEM lane
        const int t = 16 * warp + lane;                 // token row of the M=64 products
        const uint32_t lo = (uint32_t)(32 * warp) << 16;
        float *Sg = state ? state + ((size_t)n * H + h) * TC_D * TC_D : nullptr;
        // initial state slice -> TMEM (fp32) and S16 (bf16, S^T K-major)
        for (int c = 0; c < DVT; c += 16) {
            float v[16];
#pragma unroll
            for (int q = 0; q < 16; q++) v[q] = Sg ? Sg[(size_t)i * TC_D + col0 + c + q] : 0.f;
            tmem_st16(tb + lo + TM_S + c, v);
#pragma unroll
            for (int q = 0; q < 16; q++)
                stbf(S16, (uint32_t)((i >> 6) * DVT * 128) + sw128(c + q, i & 63), v[q]);
        }
        tmem_wait_st();
        fence_async_shared();
        tc_fence_before();
        mbar_arrive(&s16_ready);
        bool ok = true;
        TcChunk cd_next = nc > 0 ? chunks[c0] : TcChunk{0, 0, 0, 0};
        for (int j = 0; j < nc; j++) {
            const TcChunk cd = cd_next;
            if (j + 1 < nc) cd_next = chunks[c0 + j + 1];  // prefetched off the critical path
            const uint8_t *s = sm + (j & 1) * SB;
            if (!(ok = warp_wait_all(&x_full, j & 1, err, 0x605))) break;
            tc_fence_after();
            const float gam = reinterpret_cast<const float *>(s + OFF_GAM)[i];
            // X = U - X_acc (rows t < 16 of each warp's quarter) -> X^T in shared memory
            for (int c = 0; c < DVT; c += 16) {
                float v[16];
                tmem_ld16(tb + lo + TM_X + c, v);
                tmem_wait_ld();
                if (lane < 16) {
#pragma unroll
                    for (int q = 0; q < 16; q++) {
                        const int jj = c + q;
                        const float u = DVT == 32 ? ldbf(s + 57344, (uint32_t)(t * 64 + jj * 2))
                                                  : ldbf(s + 57344, (uint32_t)((jj >> 6) * 8192) +
                                                                        sw128(t, jj & 63));
                        stbf(XT, sw128(jj, t), u - v[q]);
                    }
                }
            }
            // S <- Gamma S, before S += Kbar^T X accumulates into it
            for (int c = 0; c < DVT; c += 16) {
                float v[16];
                tmem_ld16(tb + lo + TM_S + c, v);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 16; q++) v[q] *= gam;
                tmem_st16(tb + lo + TM_S + c, v);
            }
            tmem_wait_st();
            fence_async_shared();
            tc_fence_before();
            mbar_arrive(&xt_ready);
            if (!(ok = warp_wait_all(&done, j & 1, err, 0x606))) break;
            tc_fence_after();
            // outputs of this chunk, then the new S16
            for (int c = 0; c < DVT; c += 16) {
                float v[16];
                tmem_ld16(tb + lo + TM_O + c, v);
                tmem_wait_ld();
                if (lane < 16 && t < cd.len) {
                    uint32_t pk[8];
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
                        pk[q] = *reinterpret_cast<const uint32_t *>(&p);
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(o + ((size_t)(cd.t0 + t) * H + h) * TC_D +
                                                           col0 + c);
                    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
            }
            for (int c = 0; c < DVT; c += 16) {
                float v[16];
                tmem_ld16(tb + lo + TM_S + c, v);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 16; q++)
                    stbf(S16, (uint32_t)((i >> 6) * DVT * 128) + sw128(c + q, i & 63), v[q]);
            }
            fence_async_shared();
            tc_fence_before();
            mbar_arrive(&s16_ready);
        }
        if (ok && Sg) {
            for (int c = 0; c < DVT; c += 16) {
                float v[16];
                tmem_ld16(tb + lo + TM_S + c, v);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 16; q++) Sg[(size_t)i * TC_D + col0 + c + q] = v[q];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tmem_dealloc(tb, TM_COLS);
    }
}

// -------------------------------------------------------------------------- host side
size_t prefill_tc_block_bytes() { return PB_BYTES; }

// Launch both phases. `blocks` has room for nc * H blocks of PB_BYTES; d_table / d_c0 are
// the device copies of the chunk table and of the per-sequence first-chunk index.
int run_prefill_tc(k3cuda_ctx *ctx, float *state, void *o, const void *q, const void *k,
                   const void *v, const float *gate, const float *beta, int total_tokens,
                   int n_seq, int H, float q_scale, int gate_is_log, long long nc,
                   const void *d_table, const int *d_c0, void *blocks) {
    const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    PrepMaps pm;
    const uint64_t rs = (uint64_t)H * TC_D * 2;  // bytes per token row of q/k/v
    int rc = make_tmap_3d(&pm.q, q, BF, 2, TC_D, H, total_tokens, TC_D * 2, rs, 64, 1, 64);
    if (!rc) rc = make_tmap_3d(&pm.k, k, BF, 2, TC_D, H, total_tokens, TC_D * 2, rs, 64, 1, 64);
    if (!rc) rc = make_tmap_3d(&pm.v, v, BF, 2, TC_D, H, total_tokens, TC_D * 2, rs, 64, 1, 64);
    if (rc) return rc;
    K3_CUDA_TRY(cudaFuncSetAttribute(kda_prep_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     PS_SMEM));
    kda_prep_tc<<<dim3((unsigned)nc, (unsigned)H), 256, PS_SMEM, ctx->stream>>>(
        pm, (const TcChunk *)d_table, gate, beta, (uint8_t *)blocks, H, q_scale, gate_is_log,
        ctx->err_word);
    rc = after_launch(ctx, "kda_prep_tc");
    if (rc) return rc;

    const uint64_t nch = (uint64_t)nc * H;
    const bool wide = (long long)n_seq * H >= ctx->sm_count;
    const int dvt = wide ? 128 : 32;
    ScanMaps sm;
    uint8_t *b = (uint8_t *)blocks;
    rc = make_tmap_3d(&sm.w, b + PB_W, BF, 2, 128, 64, nch, 256, PB_BYTES, 64, 64, 1);
    if (!rc) rc = make_tmap_3d(&sm.q, b + PB_Q, BF, 2, 128, 64, nch, 256, PB_BYTES, 64, 64, 1);
    if (!rc) rc = make_tmap_3d(&sm.kb, b + PB_KB, BF, 2, 64, 128, nch, 128, PB_BYTES, 64, 128, 1);
    if (!rc) rc = make_tmap_3d(&sm.a, b + PB_A, BF, 2, 64, 64, nch, 128, PB_BYTES, 64, 64, 1);
    if (!rc)
        rc = make_tmap_3d(&sm.u, b + PB_U, BF, 2, 128, 64, nch, 256, PB_BYTES, dvt > 64 ? 64 : dvt,
                          64, 1);
    if (!rc)
        rc = make_tmap_2d(&sm.g, b + PB_G, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 128, nch, PB_BYTES,
                          128, 1);
    if (rc) return rc;
    const long long nblk = (long long)n_seq * H * (TC_D / dvt);
    if (dvt == 128) {
        const int smem = 2 * (((57344 + 128 * 128 + 512) + 1023) & ~1023) + 128 * 384 + 1024;
        K3_CUDA_TRY(cudaFuncSetAttribute(kda_scan_tc<128>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        kda_scan_tc<128><<<(unsigned)nblk, 192, smem, ctx->stream>>>(
            sm, (const TcChunk *)d_table, d_c0, (const uint8_t *)blocks, state,
            (__nv_bfloat16 *)o, H, ctx->err_word);
    } else {
        const int smem = 2 * (((57344 + 128 * 32 + 512) + 1023) & ~1023) + 32 * 384 + 1024;
        K3_CUDA_TRY(cudaFuncSetAttribute(kda_scan_tc<32>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        kda_scan_tc<32><<<(unsigned)nblk, 192, smem, ctx->stream>>>(
            sm, (const TcChunk *)d_table, d_c0, (const uint8_t *)blocks, state,
            (__nv_bfloat16 *)o, H, ctx->err_word);
    }
    return after_launch(ctx, "kda_scan_tc");
}

}  // namespace k3
