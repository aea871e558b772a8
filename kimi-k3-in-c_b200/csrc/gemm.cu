// gemm.cu -- the projections' matrix products for more than PROJ_MAXT activation rows:
// y [T][out] fp32 = x [T][in] fp32 . W [out][in]^T, the T-row form of k3_mmw
// (include/k3/k3.h:290-296: k3_matmul, src/core/k3_ops.c:265-291, and k3_matmul_bf16,
// :1122-1227, which multiply the fp32 activation by the weight exactly).
//
//   proj_gemm_tc    bf16 W, in % 64 == 0 (every projection of the released model). tcgen05
//                   with the tokens as the MMA's M (128 per tile) and 256 weight rows as N,
//                   fed by TMA through a three-stage pipeline; persistent (one CTA per SM):
//                   one thread issues the loads, one the MMAs, and four warps read the fp32
//                   accumulator out of TMEM while the next tile accumulates into the other
//                   half of TMEM.
//                   The activation arrives as its bf16 hi + lo halves (x = hi + lo to 2^-16
//                   |x|), and both halves' products accumulate into the same TMEM tile, so x
//                   is never rounded to bf16 as a whole.
//   proj_gemm_simt  fp32 W, or shapes the TMA tiles do not cover (in % 64 != 0): a shared-
//                   memory tiled product on the CUDA cores, exact fp32 products summed in fp32.
#include <algorithm>

#include "internal.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace k3 {

using namespace sm100;

constexpr int GT_M = 128, GT_N = 256, GT_K = 64, GT_NS = 3;
constexpr int GT_A = GT_M * GT_K * 2;             // 16 KB: one half of x, 128 tokens
constexpr int GT_B = GT_N * GT_K * 2;             // 32 KB: 256 weight rows
constexpr int GT_STAGE = 2 * GT_A + GT_B;         // 64 KB
constexpr int GT_SMEM = GT_NS * GT_STAGE + 1024;  // + alignment slack

struct GemmMaps {
    CUtensorMap x;  // [2][T][in] bf16 (hi, lo), box 64 x 128 x 1
    CUtensorMap w;  // [out][in] bf16, box 64 x 256
};

__device__ __forceinline__ bool all_wait(uint64_t *bar, uint32_t parity, unsigned *err,
                                         unsigned code) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code));
}

// Persistent: one CTA per SM walks the tiles tau = CTA, CTA + grid, ...; tile tau covers tokens
// [128 m, +128) x weight rows [256 n, +256) with m = tau % m_tiles (the token tiles vary
// fastest, so the CTAs that share a weight tile run together and the weight streams from DRAM
// about once while x, a few tens of MB, stays in L2). Warp 0 issues the TMA loads, warp 1 the
// MMAs, warps 2-5 drain the fp32 accumulator: TMEM holds two 256-column accumulators, so the
// epilogue of one tile runs under the MMAs of the next. Rows past T or out are zero-filled by
// TMA and never stored.
constexpr int GT_THREADS = 192;

__global__ void __launch_bounds__(GT_THREADS, 1)
proj_gemm_tc(const __grid_constant__ GemmMaps maps, float *__restrict__ y, int T, int in,
             int out, int m_tiles, int n_tiles, unsigned *__restrict__ err) {
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar_full[GT_NS], bar_empty[GT_NS], acc_full[2], acc_empty[2];
    __shared__ uint32_t tslot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int KB = in / GT_K, ntile = m_tiles * n_tiles;
    if (tid == 0) {
        for (int i = 0; i < GT_NS; i++) {
            mbar_init(&bar_full[i], 1);
            mbar_init(&bar_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
        }
        fence_barrier_init();
        prefetch_tmap(&maps.x);
        prefetch_tmap(&maps.w);
    }
    if (warp == 2) tmem_alloc(&tslot, 2 * GT_N);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tslot;

    if (warp == 0 && lane == 0) {
        // producer: stage it % NS holds x hi, x lo and the weight block of the it-th K block
        // this CTA loads (counting across its tiles)
        long long it = 0;
        int last[GT_NS];
        for (int st = 0; st < GT_NS; st++) last[st] = -1;
        bool ok = true;
        for (int tau = blockIdx.x; tau < ntile && ok; tau += gridDim.x) {
            const int t0 = (tau % m_tiles) * GT_M, n0 = (tau / m_tiles) * GT_N;
            for (int kb = 0; kb < KB; kb++, it++) {
                const int st = (int)(it % GT_NS);
                const long long use = it / GT_NS;
                if (use > 0 && !(ok = mbar_wait(&bar_empty[st], (uint32_t)((use - 1) & 1), err,
                                                0x601)))
                    break;
                uint8_t *s = sm + st * GT_STAGE;
                mbar_expect_tx(&bar_full[st], GT_STAGE);
                tma_load_3d(s, &maps.x, &bar_full[st], kb * GT_K, t0, 0);
                tma_load_3d(s + GT_A, &maps.x, &bar_full[st], kb * GT_K, t0, 1);
                tma_load_2d(s + 2 * GT_A, &maps.w, &bar_full[st], kb * GT_K, n0);
                last[st] = (int)(use & 1);
            }
        }
        // every load issued has landed before the CTA may exit
        for (int st = 0; st < GT_NS; st++)
            if (last[st] >= 0) mbar_wait_quiet(&bar_full[st], (uint32_t)last[st]);
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: accumulator lt & 1 of the lt-th tile, D[128 tokens][256 rows] +=
        // (x_hi + x_lo) . W^T, K = 16 per instruction
        constexpr uint32_t id = idesc_f16(GT_M, GT_N, false, false);
        long long it = 0;
        int lt = 0;
        bool ok = true;
        for (int tau = blockIdx.x; tau < ntile && ok; tau += gridDim.x, lt++) {
            const int ab = lt & 1;
            const uint32_t d = tb + (uint32_t)(ab * GT_N);
            if (lt >= 2 && !(ok = mbar_wait(&acc_empty[ab], (uint32_t)(((lt >> 1) - 1) & 1), err,
                                            0x604)))
                break;
            tc_fence_after();
            for (int kb = 0; kb < KB; kb++, it++) {
                const int st = (int)(it % GT_NS);
                if (!(ok = mbar_wait(&bar_full[st], (uint32_t)((it / GT_NS) & 1), err, 0x602)))
                    break;
                tc_fence_after();
                const uint32_t s = smem_u32(sm + st * GT_STAGE);
#pragma unroll
                for (int kin = 0; kin < GT_K / 16; kin++) {
                    const uint64_t bd = sdesc_kmajor(s + 2 * GT_A + kin * 32);
                    mma_bf16_ss(d, sdesc_kmajor(s + kin * 32), bd, id, (kb | kin) ? 1u : 0u);
                    mma_bf16_ss(d, sdesc_kmajor(s + GT_A + kin * 32), bd, id, 1u);
                }
                mma_commit(&bar_empty[st]);  // the stage is free once these MMAs have read it
            }
            if (ok) mma_commit(&acc_full[ab]);  // the tile's accumulator is complete
        }
    } else if (warp >= 2) {
        // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its lane quarter)
        const int q4 = warp & 3;
        const bool vec = (out & 3) == 0;
        int lt = 0;
        for (int tau = blockIdx.x; tau < ntile; tau += gridDim.x, lt++) {
            const int ab = lt & 1;
            const int t0 = (tau % m_tiles) * GT_M, n0 = (tau / m_tiles) * GT_N;
            if (!all_wait(&acc_full[ab], (uint32_t)((lt >> 1) & 1), err, 0x603)) break;
            tc_fence_after();
            const int t = t0 + 32 * q4 + lane;
            for (int c = 0; c < GT_N; c += 16) {
                if (n0 + c >= out) break;
                float v[16];
                tmem_ld16(tb + ((uint32_t)(32 * q4) << 16) + (uint32_t)(ab * GT_N + c), v);
                tmem_wait_ld();
                if (t < T) {
                    float *dst = y + (size_t)t * out + n0 + c;
                    if (vec && n0 + c + 16 <= out) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4)
                            *reinterpret_cast<float4 *>(dst + i) =
                                make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            if (n0 + c + i < out) dst[i] = v[i];
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[ab]);  // this accumulator may take the tile after next
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        __syncwarp();
        tmem_dealloc(tb, 2 * GT_N);
    }
}

// ------------------------------------------------------------------------- CUDA cores
constexpr int GS_T = 64, GS_O = 64, GS_K = 32;

// Block (o-tile, t-tile): 256 threads, each 4 tokens x 4 weight rows, K in slices of 32
// staged in shared memory (transposed so each thread's operands are contiguous).
template <typename WT>
__global__ void __launch_bounds__(256)
proj_gemm_simt(float *__restrict__ y, const float *__restrict__ x, const WT *__restrict__ W,
               int T, int in, int out) {
    __shared__ float xs[GS_K][GS_T + 4];
    __shared__ float ws[GS_K][GS_O + 4];
    const int o0 = blockIdx.x * GS_O, t0 = blockIdx.y * GS_T, tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;  // rows o0 + 4 tx .., tokens t0 + 4 ty ..
    float acc[4][4] = {};
    for (int k0 = 0; k0 < in; k0 += GS_K) {
        for (int e = tid; e < GS_T * GS_K; e += 256) {
            const int r = e / GS_K, k = e % GS_K;
            const int t = t0 + r, o = o0 + r, kk = k0 + k;
            xs[k][r] = (t < T && kk < in) ? x[(size_t)t * in + kk] : 0.f;
            ws[k][r] = (o < out && kk < in) ? io<WT>::ld(W + (size_t)o * in + kk) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < GS_K; k++) {
            const float4 a = *reinterpret_cast<const float4 *>(&xs[k][4 * ty]);
            const float4 b = *reinterpret_cast<const float4 *>(&ws[k][4 * tx]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int t = t0 + 4 * ty + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int o = o0 + 4 * tx + j;
            if (o < out) y[(size_t)t * out + o] = acc[i][j];
        }
    }
}

// y [T][out] = x [T][in] W^T. xs: x's bf16 hi/lo halves ([2][T][in]) when W is bf16 (the
// tensor-core path reads them); may be null otherwise.
int gemm(k3cuda_ctx *ctx, float *y, const float *x, const __nv_bfloat16 *xs, const void *W,
         int wdt, int T, int in, int out) {
    if (T <= 0 || out <= 0) return K3CUDA_OK;
    const bool tc = wdt == K3CUDA_BF16 && xs && in >= GT_K && in % GT_K == 0 && aligned(xs, 16) &&
                    aligned(W, 16);
    if (tc) {
        GemmMaps maps;
        const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        int rc = make_tmap_3d(&maps.x, xs, BF, 2, (uint64_t)in, (uint64_t)T, 2,
                              (uint64_t)in * 2, (uint64_t)T * in * 2, GT_K, GT_M, 1);
        if (!rc)
            rc = make_tmap_2d(&maps.w, W, BF, 2, (uint64_t)in, (uint64_t)out, (uint64_t)in * 2,
                              GT_K, GT_N);
        if (rc) return rc;
        if ((rc = set_smem(proj_gemm_tc, GT_SMEM))) return rc;
        const int m_tiles = (T + GT_M - 1) / GT_M, n_tiles = (out + GT_N - 1) / GT_N;
        const int grid = std::min(m_tiles * n_tiles, ctx->sm_count);
        proj_gemm_tc<<<grid, GT_THREADS, GT_SMEM, ctx->stream>>>(maps, y, T, in, out, m_tiles,
                                                                 n_tiles, ctx->err_word);
        return after_launch(ctx, "proj_gemm_tc");
    }
    const dim3 grid((out + GS_O - 1) / GS_O, (T + GS_T - 1) / GS_T);
    if (wdt == K3CUDA_BF16)
        proj_gemm_simt<__nv_bfloat16><<<grid, 256, 0, ctx->stream>>>(
            y, x, (const __nv_bfloat16 *)W, T, in, out);
    else
        proj_gemm_simt<float><<<grid, 256, 0, ctx->stream>>>(y, x, (const float *)W, T, in, out);
    return after_launch(ctx, "proj_gemm_simt");
}

}  // namespace k3
