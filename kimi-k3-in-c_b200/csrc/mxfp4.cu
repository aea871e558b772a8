// mxfp4.cu -- MXFP4 expert projections on the device: k3_matmul_mxfp4 and k3_mxfp4_dequant
// (src/core/k3_ops.c:1394-1831; format include/k3/k3.h:523-569).
//
// Format: packed [rows][in/2] bytes, two E2M1 codes per byte with the LOW nibble the EVEN
// element; scales [rows][in/group] E8M0 bytes; w = E2M1[code] * 2^(scale - 127), scale 255
// read as 0. The reference multiplies fp32 x by these weights exactly and sums in double.
//
// Decode (T <= 4 activation rows): the expert's bytes are streamed once. A 16-byte load is
// exactly one 32-element group with one scale byte. sm_100a converts a byte of two E2M1
// codes to an f16 pair in one instruction (cvt.rn.f16x2.e2m1x2; every E2M1 value is exact
// in f16), the pair is widened to fp32, and the group's 32 products are summed by fused
// multiply-adds before the power-of-two scale is applied once (exact, as the reference's
// scale folding).
//
// More rows of x (a prefill's tokens routed to one expert): the weights are expanded to
// bf16 (exact: 3 significant bits and an fp32-range exponent) and multiplied on tcgen05
// (gemm.cu) against x split into bf16 hi + lo halves, the same near-fp32 scheme as the bf16
// trunk.
#include <cuda_fp16.h>

#include "internal.cuh"

namespace k3 {

constexpr int FP4_THREADS = 256, FP4_WARPS = 8, FP4_MAXT = 4, FP4_GROUP = 32;

__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// the eight E2M1 codes of a 32-bit word as fp32, element order (low nibble first)
__device__ __forceinline__ void e2m1x8(unsigned int word, float w[8]) {
    unsigned int h[4];
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
        : "r"(word));
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h[j]));
        w[2 * j] = f.x;
        w[2 * j + 1] = f.y;
    }
}

// 2^(s - 127) as fp32 (s = 0 is the subnormal 2^-127), 255 (NaN by the spec) as 0
__device__ __forceinline__ float e8m0(unsigned int s) {
    return s == 255u ? 0.f : s == 0u ? __uint_as_float(0x00400000u) : __uint_as_float(s << 23);
}

constexpr int FP4_MAXSEG = 64;  // matrices of one launch (16 experts x w1, w3 is 32)

struct Fp4Args {
    const unsigned char *packed[FP4_MAXSEG], *scales[FP4_MAXSEG];
    const float *x[FP4_MAXSEG];  // [T][in] each
    float *y[FP4_MAXSEG];        // [T][rows] each
    int in, rows, ks, blocks_per_seg;
};

// A warp owns R rows and one of `ks` slices of the groups; lane l takes groups l, l+32, ...
// of every row (16 bytes = one 32-element group per load, 512 contiguous bytes per row per
// warp load), and each x load serves all R rows. R = 8 measured best for the experts'
// 1.8 KB rows (more bytes in flight per warp); the ks slices are summed in shared memory in
// a fixed order.
template <int NT, int R>
__global__ void __launch_bounds__(FP4_THREADS) mxfp4_rows(const __grid_constant__ Fp4Args a) {
    __shared__ float part[FP4_WARPS][R * NT];
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seg = blockIdx.x / a.blocks_per_seg, b = blockIdx.x - seg * a.blocks_per_seg;
    const float *xs = a.x[seg];
    const int ks = a.ks, rg = warp / ks, sl = warp - rg * ks;
    const int row0 = (b * (FP4_WARPS / ks) + rg) * R;
    const int ngrp = a.in / FP4_GROUP, per = (ngrp + ks - 1) / ks;
    const int g0 = sl * per, g1 = min(ngrp, g0 + per);
    // rows past the end re-read the last row and are never stored
    const int nr = max(1, min(R, a.rows - row0));
    const unsigned char *pbase = a.packed[seg] + (size_t)min(row0, a.rows - 1) * (a.in / 2);
    const unsigned char *sbase = a.scales[seg] + (size_t)min(row0, a.rows - 1) * ngrp;
    const size_t pstride = a.in / 2;
    float acc[R][NT];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[r][t] = 0.f;
    uint4 pk[R];
    float sf[R];
    auto load_w = [&](int g) {  // this lane's group g of every row: codes and scale
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int rr = r < nr ? r : nr - 1;
            pk[r] = ld_stream16(pbase + rr * pstride + (size_t)g * 16);
            sf[r] = e8m0(__ldg(sbase + (size_t)rr * ngrp + g));
        }
    };
    // the first group's weights are fetched before waiting for the previous kernel (which
    // produced x, never the weights)
    if (g0 + lane < g1) load_w(g0 + lane);
    pdl_wait();
#pragma unroll 1
    for (int g = g0 + lane; g < g1; g += 32) {
        if (g != g0 + lane) load_w(g);
        float gs[R][NT];
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int t = 0; t < NT; t++) gs[r][t] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {  // 8 elements per 32-bit word
            float xv[NT][8];
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float4 *xp =
                    reinterpret_cast<const float4 *>(xs + (size_t)t * a.in + (size_t)g * 32 + 8 * j);
                const float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
                xv[t][0] = x0.x; xv[t][1] = x0.y; xv[t][2] = x0.z; xv[t][3] = x0.w;
                xv[t][4] = x1.x; xv[t][5] = x1.y; xv[t][6] = x1.z; xv[t][7] = x1.w;
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
                float w[8];
                e2m1x8(j == 0 ? pk[r].x : j == 1 ? pk[r].y : j == 2 ? pk[r].z : pk[r].w, w);
#pragma unroll
                for (int t = 0; t < NT; t++)
#pragma unroll
                    for (int e = 0; e < 8; e++) gs[r][t] = fmaf(w[e], xv[t][e], gs[r][t]);
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int t = 0; t < NT; t++) acc[r][t] = fmaf(gs[r][t], sf[r], acc[r][t]);
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) {
            float v = acc[r][t];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) part[warp][r * NT + t] = v;
        }
    __syncthreads();
    for (int i = lane; i < R * NT; i += 32) {
        if (sl != 0) break;
        const int r = i / NT, t = i - r * NT;
        float v = 0.f;
        for (int j = 0; j < ks; j++) v += part[rg * ks + j][i];
        if (row0 + r < a.rows) a.y[seg][(size_t)t * a.rows + row0 + r] = v;
    }
}

// out[r][i] = E2M1 * 2^(s-127) as fp32 or bf16 (exact in both), one byte (two elements) per
// thread; any even `in` and any group.
template <typename OUT>
__global__ void mxfp4_dequant_k(OUT *__restrict__ out, const unsigned char *__restrict__ packed,
                                const unsigned char *__restrict__ scales, int rows, int in,
                                int group) {
    const long long nbytes = (long long)rows * (in / 2);
    const int ngrp = (in + group - 1) / group;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nbytes;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / (in / 2)), c = (int)(i - (long long)r * (in / 2));
        unsigned int h;
        const unsigned short b = packed[i];
        asm("{\n\t.reg .b8 t;\n\tcvt.u8.u16 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
            : "=r"(h) : "h"(b));
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h));
        const size_t o = (size_t)r * in + 2 * (size_t)c;
        const float s0 = e8m0(scales[(size_t)r * ngrp + (2 * c) / group]);
        const float s1 = e8m0(scales[(size_t)r * ngrp + (2 * c + 1) / group]);
        io<OUT>::st(out + o, f.x * s0);
        io<OUT>::st(out + o + 1, f.y * s1);
    }
}

static int dequant(k3cuda_ctx *ctx, void *out, int out_dtype, const unsigned char *packed,
                   const unsigned char *scales, int rows, int in, int group) {
    const long long nbytes = (long long)rows * (in / 2);
    if (nbytes == 0) return K3CUDA_OK;
    const long long want = (nbytes + 255) / 256;
    const int blocks = (int)(want < 16LL * ctx->sm_count ? want : 16LL * ctx->sm_count);
    if (out_dtype == K3CUDA_BF16)
        mxfp4_dequant_k<__nv_bfloat16><<<blocks, 256, 0, ctx->stream>>>(
            (__nv_bfloat16 *)out, packed, scales, rows, in, group);
    else
        mxfp4_dequant_k<float><<<blocks, 256, 0, ctx->stream>>>((float *)out, packed, scales, rows,
                                                                in, group);
    return after_launch(ctx, "mxfp4_dequant");
}

static size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

static bool streaming_path(int T, int in, int group, const void *packed) {
    return T <= FP4_MAXT && group == FP4_GROUP && in % FP4_GROUP == 0 && aligned(packed, 16);
}

static int check_fp4(int in, int rows, int group, int T) {
    K3_ARG_CHECK(in >= 2 && rows >= 0 && T >= 0, "mxfp4: in=%d rows=%d T=%d", in, rows, T);
    K3_ARG_CHECK(!(in & 1), "mxfp4: in=%d is odd (two elements per byte)", in);
    K3_ARG_CHECK(group >= 2 && group <= 64 && !(group & 1), "mxfp4: group=%d outside [2, 64]",
                 group);
    return K3CUDA_OK;
}

}  // namespace k3

using namespace k3;

extern "C" int k3cuda_mxfp4_dequant(k3cuda_ctx *ctx, void *out, int out_dtype,
                                    const unsigned char *packed, const unsigned char *scales,
                                    int rows, int in, int group) {
    int rc = enter(ctx);
    if (rc) return rc;
    if ((rc = check_fp4(in, rows, group, 1))) return rc;
    K3_ARG_CHECK(out_dtype == K3CUDA_F32 || out_dtype == K3CUDA_BF16, "bad out_dtype");
    if (rows == 0) return K3CUDA_OK;
    K3_ARG_CHECK(out && packed && scales, "mxfp4_dequant: null pointer");
    return dequant(ctx, out, out_dtype, packed, scales, rows, in, group);
}

extern "C" int k3cuda_matmul_mxfp4_workspace(int T, int in, int rows, int group, size_t *bytes) {
    K3_ARG_CHECK(bytes, "null bytes");
    int rc = check_fp4(in, rows, group, T);
    if (rc) return rc;
    // the streaming path needs none; the GEMM path the bf16 weights and x's hi/lo split
    *bytes = T <= FP4_MAXT && group == FP4_GROUP && in % FP4_GROUP == 0
                 ? 0
                 : a256((size_t)rows * in * 2) + a256((size_t)2 * T * in * 2);
    return K3CUDA_OK;
}

// rows per warp: 8 for one or two activation rows, 4 beyond (registers)
template <int NT> constexpr int fp4_rows() { return NT <= 2 ? 8 : 4; }

template <int NT>
static int launch_fp4(k3cuda_ctx *ctx, const Fp4Args &a, int blocks) {
    return launch_pdl(ctx, ctx->stream, "mxfp4_rows", mxfp4_rows<NT, fp4_rows<NT>()>,
                      dim3(blocks), dim3(FP4_THREADS), 0, a);
}

// The streaming kernel over n matrices of one shape (T <= 4, group 32, in % 32 == 0).
static int stream_fp4(k3cuda_ctx *ctx, const unsigned char *const *packed,
                      const unsigned char *const *scales, const float *const *x,
                      float *const *y, int n, int in, int rows, int T) {
    Fp4Args a{};
    for (int i = 0; i < n; i++) {
        a.packed[i] = packed[i];
        a.scales[i] = scales[i];
        a.x[i] = x[i];
        a.y[i] = y[i];
    }
    a.in = in;
    a.rows = rows;
    const int R = T <= 2 ? fp4_rows<1>() : fp4_rows<4>();
    const int ngrp = in / FP4_GROUP;
    auto per_seg = [&](int ks) {
        const int per_block = (FP4_WARPS / ks) * R;
        return (rows + per_block - 1) / per_block;
    };
    // split the groups over up to 4 warps while the grid is short of ~8 blocks per SM and
    // every slice keeps at least two groups per lane
    int ks = 1;
    while (ks < 4 && (long long)n * per_seg(ks) < 8LL * ctx->sm_count && ngrp / (2 * ks) >= 64)
        ks *= 2;
    a.ks = ks;
    a.blocks_per_seg = per_seg(ks);
    const long long blocks = (long long)n * a.blocks_per_seg;
    if (blocks > 0x7fffffffLL) return set_error(K3CUDA_ERR_ARG, "matmul_mxfp4: grid too large");
    switch (T) {
        case 1: return launch_fp4<1>(ctx, a, (int)blocks);
        case 2: return launch_fp4<2>(ctx, a, (int)blocks);
        case 3: return launch_fp4<3>(ctx, a, (int)blocks);
        default: return launch_fp4<4>(ctx, a, (int)blocks);
    }
}

extern "C" int k3cuda_matmul_mxfp4(k3cuda_ctx *ctx, float *y, const float *x,
                                   const unsigned char *packed, const unsigned char *scales,
                                   int in, int rows, int group, int T, void *workspace,
                                   size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    if ((rc = check_fp4(in, rows, group, T))) return rc;
    if (T == 0 || rows == 0) return K3CUDA_OK;
    K3_ARG_CHECK(y && x && packed && scales, "matmul_mxfp4: null pointer");
    K3_ARG_CHECK(aligned(x, 16) && aligned(y, 16), "matmul_mxfp4: x and y must be 16-byte aligned");
    if (streaming_path(T, in, group, packed))
        return stream_fp4(ctx, &packed, &scales, &x, &y, 1, in, rows, T);
    size_t need = 0;
    if ((rc = k3cuda_matmul_mxfp4_workspace(T, in, rows, group, &need))) return rc;
    if (workspace_bytes < need || !workspace)
        return set_error(K3CUDA_ERR_WORKSPACE, "matmul_mxfp4: workspace %zu < %zu bytes",
                         workspace_bytes, need);
    K3_ARG_CHECK(aligned(workspace, 256), "matmul_mxfp4: workspace must be 256-byte aligned");
    __nv_bfloat16 *wb = (__nv_bfloat16 *)workspace;
    __nv_bfloat16 *xs = (__nv_bfloat16 *)((char *)workspace + a256((size_t)rows * in * 2));
    if ((rc = dequant(ctx, wb, K3CUDA_BF16, packed, scales, rows, in, group))) return rc;
    if ((rc = split(ctx, xs, x, (long long)T * in))) return rc;
    return gemm(ctx, y, x, xs, wb, K3CUDA_BF16, T, in, rows);
}

extern "C" int k3cuda_matmul_mxfp4_batch(k3cuda_ctx *ctx, float *const *y,
                                         const float *const *x,
                                         const unsigned char *const *packed,
                                         const unsigned char *const *scales, int n, int in,
                                         int rows, int T) {
    int rc = enter(ctx);
    if (rc) return rc;
    if ((rc = check_fp4(in, rows, FP4_GROUP, T))) return rc;
    K3_ARG_CHECK(n >= 0 && n <= FP4_MAXSEG, "matmul_mxfp4_batch: n=%d outside [0, %d]", n,
                 FP4_MAXSEG);
    if (n == 0 || T == 0 || rows == 0) return K3CUDA_OK;
    K3_ARG_CHECK(y && x && packed && scales, "matmul_mxfp4_batch: null pointer array");
    if (T > FP4_MAXT || in % FP4_GROUP)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "matmul_mxfp4_batch: T=%d in=%d (needs T <= %d, "
                         "in %% 32 == 0; use k3cuda_matmul_mxfp4 per matrix)", T, in, FP4_MAXT);
    for (int i = 0; i < n; i++)
        K3_ARG_CHECK(y[i] && x[i] && packed[i] && scales[i] && aligned(y[i], 16) &&
                         aligned(x[i], 16) && aligned(packed[i], 16),
                     "matmul_mxfp4_batch: matrix %d: null or not 16-byte aligned", i);
    return stream_fp4(ctx, packed, scales, x, y, n, in, rows, T);
}
