// mla_decode.cu -- absorbed MLA decode over the compressed latent cache.
//
// Replaces the per-head attention loop of k3_mla_cached (reference src/core/k3_ops.c:
// 381-411) for one query token per sequence. The reference caches the EXPANDED keys and
// values (k3_ops.c:304-315, 351-367); here the cache holds the latent c_s (kv_lora wide)
// and the shared rope slot r_s, and the per-head blocks of kv_b are folded into the query
// and the output instead:
//     q_lat  = W_UK^T q_nope                          (mla_q_absorb)
//     score  = (q_lat . c_s + q_rope . r_s) * scale   (mla_attend_split, split-K over s)
//     p      = softmax(score) (fp32, max-subtracted)  (mla_attend_split)
//     o_lat  = sum_s p_s c_s                          (mla_attend_split)
//     out    = W_UV o_lat                             (mla_merge_project)
// Split-K: each CTA covers a slice of the context and writes (max, sum, o_lat) per head;
// the merge rescales the slices to a common max, exactly the flash-decoding identity.
#include <algorithm>
#include <vector>

#include "internal.cuh"

namespace k3 {

constexpr int MLA_DN = 128, MLA_DR = 64, MLA_DL = 512, MLA_DV = 128;
constexpr int MLA_QW = MLA_DL + MLA_DR;  // 576: absorbed query width
constexpr int MLA_SPLIT = 1024;          // context tokens per split CTA
constexpr int MLA_TILE = 32;             // tokens per shared-memory tile
constexpr int MLA_HG = 32;               // heads per split CTA

__device__ __forceinline__ float bf(const __nv_bfloat16 *p) { return __bfloat162float(*p); }

// q_lat[b][h][0:512] = W_UK[h]^T q_nope[b][h]; q_lat[b][h][512:576] = q_rope[b][h].
// One CTA per (head, group of 16 sequences); thread l owns latent columns l and l+256.
__global__ void __launch_bounds__(256)
mla_q_absorb(const __nv_bfloat16 *__restrict__ q_nope, const __nv_bfloat16 *__restrict__ q_rope,
             const __nv_bfloat16 *__restrict__ w_uk, float *__restrict__ qabs, int B, int H) {
    __shared__ float sq[16][MLA_DN];
    const int h = blockIdx.x, b0 = blockIdx.y * 16, tid = threadIdx.x;
    for (int e = tid; e < 16 * MLA_DN; e += 256) {
        const int bb = e / MLA_DN, i = e % MLA_DN;
        sq[bb][i] = (b0 + bb < B) ? bf(q_nope + ((size_t)(b0 + bb) * H + h) * MLA_DN + i) : 0.f;
    }
    __syncthreads();
    float acc0[16], acc1[16];
#pragma unroll
    for (int bb = 0; bb < 16; bb++) acc0[bb] = acc1[bb] = 0.f;
    const __nv_bfloat16 *W = w_uk + (size_t)h * MLA_DN * MLA_DL;
    for (int i = 0; i < MLA_DN; i++) {
        const float w0 = bf(W + (size_t)i * MLA_DL + tid), w1 = bf(W + (size_t)i * MLA_DL + tid + 256);
#pragma unroll
        for (int bb = 0; bb < 16; bb++) {
            acc0[bb] += sq[bb][i] * w0;
            acc1[bb] += sq[bb][i] * w1;
        }
    }
    for (int bb = 0; bb < 16 && b0 + bb < B; bb++) {
        float *dst = qabs + ((size_t)(b0 + bb) * H + h) * MLA_QW;
        dst[tid] = acc0[bb];
        dst[tid + 256] = acc1[bb];
        if (tid < MLA_DR) dst[MLA_DL + tid] = bf(q_rope + ((size_t)(b0 + bb) * H + h) * MLA_DR + tid);
    }
}

struct SplitDesc {
    int b, s0, s1, slot;
};

// One CTA per (split, head group): online softmax over its context slice for 32 heads.
__global__ void __launch_bounds__(256, 1)
mla_attend_split(const SplitDesc *__restrict__ splits, const float *__restrict__ qabs,
                 const __nv_bfloat16 *__restrict__ latent, const __nv_bfloat16 *__restrict__ rope,
                 float *__restrict__ part, int H, int cap, float scale) {
    extern __shared__ __align__(16) float sm[];
    float *sQ = sm;                              // [MLA_HG][576]
    float *sC = sQ + MLA_HG * MLA_QW;            // [MLA_TILE][576]
    float *sP = sC + MLA_TILE * MLA_QW;          // [MLA_HG][MLA_TILE]
    float *sM = sP + MLA_HG * MLA_TILE;          // [MLA_HG] running max
    float *sL = sM + MLA_HG;                     // [MLA_HG] running sum
    float *sF = sL + MLA_HG;                     // [MLA_HG] rescale factor of this tile
    const SplitDesc sd = splits[blockIdx.x];
    const int hg = blockIdx.y, h0 = hg * MLA_HG, tid = threadIdx.x;
    const int nh = min(MLA_HG, H - h0);
    for (int e = tid; e < MLA_HG * MLA_QW; e += 256) {
        const int hh = e / MLA_QW, c = e % MLA_QW;
        sQ[e] = hh < nh ? qabs[((size_t)sd.b * H + h0 + hh) * MLA_QW + c] : 0.f;
    }
    if (tid < MLA_HG) { sM[tid] = -INFINITY; sL[tid] = 0.f; }
    float acc[MLA_HG][2];
#pragma unroll
    for (int hh = 0; hh < MLA_HG; hh++) acc[hh][0] = acc[hh][1] = 0.f;

    for (int s0 = sd.s0; s0 < sd.s1; s0 += MLA_TILE) {
        const int nt = min(MLA_TILE, sd.s1 - s0);
        __syncthreads();
        for (int e = tid; e < MLA_TILE * MLA_QW; e += 256) {
            const int s = e / MLA_QW, c = e % MLA_QW;
            float x = 0.f;
            if (s < nt) {
                const size_t pos = (size_t)sd.b * cap + s0 + s;
                x = c < MLA_DL ? bf(latent + pos * MLA_DL + c) : bf(rope + pos * MLA_DR + c - MLA_DL);
            }
            sC[e] = x;
        }
        __syncthreads();
        // scores: 4 (head, token) pairs per thread
        for (int e = tid; e < MLA_HG * MLA_TILE; e += 256) {
            const int hh = e / MLA_TILE, s = e % MLA_TILE;
            float d = 0.f;
            const float *qq = sQ + hh * MLA_QW, *cc = sC + s * MLA_QW;
            for (int c = 0; c < MLA_QW; c++) d += qq[c] * cc[c];
            sP[e] = s < nt ? d * scale : -INFINITY;
        }
        __syncthreads();
        if (tid < MLA_HG) {
            float mx = sM[tid];
            for (int s = 0; s < nt; s++) mx = fmaxf(mx, sP[tid * MLA_TILE + s]);
            const float f = expf(sM[tid] - mx);
            float l = sL[tid] * f;
            for (int s = 0; s < MLA_TILE; s++) {
                const float p = s < nt ? expf(sP[tid * MLA_TILE + s] - mx) : 0.f;
                sP[tid * MLA_TILE + s] = p;
                l += p;
            }
            sM[tid] = mx;
            sL[tid] = l;
            sF[tid] = f;
        }
        __syncthreads();
#pragma unroll
        for (int hh = 0; hh < MLA_HG; hh++) {
            const float f = sF[hh];
            float a0 = acc[hh][0] * f, a1 = acc[hh][1] * f;
            for (int s = 0; s < nt; s++) {
                const float p = sP[hh * MLA_TILE + s];
                a0 += p * sC[s * MLA_QW + tid];
                a1 += p * sC[s * MLA_QW + tid + 256];
            }
            acc[hh][0] = a0;
            acc[hh][1] = a1;
        }
    }
    __syncthreads();
    for (int hh = 0; hh < nh; hh++) {
        float *dst = part + ((size_t)sd.slot * H + h0 + hh) * (MLA_DL + 2);
        dst[tid] = acc[hh][0];
        dst[tid + 256] = acc[hh][1];
        if (tid == 0) { dst[MLA_DL] = sM[hh]; dst[MLA_DL + 1] = sL[hh]; }
    }
}

// One CTA per (sequence, head): merge the split partials, then out = W_UV o_lat.
template <typename OUT>
__global__ void __launch_bounds__(128)
mla_merge_project(const float *__restrict__ part, const int *__restrict__ slot0,
                  const __nv_bfloat16 *__restrict__ w_uv, OUT *__restrict__ out, int H) {
    __shared__ float so[MLA_DL];
    const int b = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int p0 = slot0[b], p1 = slot0[b + 1];
    const size_t stride = (size_t)H * (MLA_DL + 2);
    const float *base = part + (size_t)h * (MLA_DL + 2);
    float mx = -INFINITY;
    for (int p = p0; p < p1; p++) mx = fmaxf(mx, base[p * stride + MLA_DL]);
    float l = 0.f;
    for (int p = p0; p < p1; p++)
        l += expf(base[p * stride + MLA_DL] - mx) * base[p * stride + MLA_DL + 1];
    const float inv = 1.f / l;
    for (int c = tid; c < MLA_DL; c += 128) {
        float a = 0.f;
        for (int p = p0; p < p1; p++) a += expf(base[p * stride + MLA_DL] - mx) * base[p * stride + c];
        so[c] = a * inv;
    }
    __syncthreads();
    const __nv_bfloat16 *W = w_uv + (size_t)h * MLA_DV * MLA_DL;
    for (int j = warp; j < MLA_DV; j += 4) {
        float a = 0.f;
        for (int c = lane; c < MLA_DL; c += 32) a += bf(W + (size_t)j * MLA_DL + c) * so[c];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
        if (lane == 0) io<OUT>::st(out + ((size_t)b * H + h) * MLA_DV + j, a);
    }
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct MlaPlan {
    std::vector<SplitDesc> splits;
    std::vector<int> slot0;
};

static void plan(const int *ctx_lens, int B, MlaPlan &p) {
    p.splits.clear();
    p.slot0.assign((size_t)B + 1, 0);
    int slot = 0;
    for (int b = 0; b < B; b++) {
        p.slot0[b] = slot;
        for (int s = 0; s < ctx_lens[b]; s += MLA_SPLIT)
            p.splits.push_back(SplitDesc{b, s, std::min(ctx_lens[b], s + MLA_SPLIT), slot++});
    }
    p.slot0[B] = slot;
}

static size_t ws_bytes(int nsplit, int B, int H) {
    return align256((size_t)nsplit * sizeof(SplitDesc)) + align256((size_t)(B + 1) * sizeof(int)) +
           align256((size_t)B * H * MLA_QW * sizeof(float)) +
           align256((size_t)nsplit * H * (MLA_DL + 2) * sizeof(float));
}

}  // namespace k3

using namespace k3;

extern "C" int k3cuda_mla_decode_workspace(const int *ctx_lens, int B, int H, int dl, int dv,
                                           size_t *bytes) {
    K3_ARG_CHECK(bytes && ctx_lens && B >= 0 && H >= 1 && H <= 128, "bad MLA workspace query");
    if (dl != MLA_DL || dv != MLA_DV)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "mla_decode: dl=%d dv=%d not built", dl, dv);
    for (int b = 0; b < B; b++)
        K3_ARG_CHECK(ctx_lens[b] >= 1, "ctx_lens[%d]=%d must be >= 1", b, ctx_lens[b]);
    MlaPlan p;
    plan(ctx_lens, B, p);
    *bytes = ws_bytes((int)p.splits.size(), B, H);
    return K3CUDA_OK;
}

extern "C" int k3cuda_mla_decode(k3cuda_ctx *ctx, void *out, int out_dtype, const void *q_nope,
                                 const void *q_rope, const void *latent, const void *rope,
                                 const void *w_uk, const void *w_uv, const int *ctx_lens, int B,
                                 int cap, int H, int dn, int dr, int dl, int dv, float scale,
                                 void *workspace, size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (dn != MLA_DN || dr != MLA_DR || dl != MLA_DL || dv != MLA_DV)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "mla_decode: dn=%d dr=%d dl=%d dv=%d not built",
                         dn, dr, dl, dv);
    K3_ARG_CHECK(out_dtype == K3CUDA_F32 || out_dtype == K3CUDA_BF16, "bad out_dtype");
    K3_ARG_CHECK(H >= 1 && H <= 128 && B >= 0, "bad H=%d B=%d", H, B);
    if (B == 0) return K3CUDA_OK;
    K3_ARG_CHECK(ctx_lens, "null ctx_lens");
    for (int b = 0; b < B; b++)
        K3_ARG_CHECK(ctx_lens[b] >= 1 && ctx_lens[b] <= cap, "ctx_lens[%d]=%d outside [1, %d]", b,
                     ctx_lens[b], cap);
    K3_ARG_CHECK(out && q_nope && q_rope && latent && rope && w_uk && w_uv, "null pointer");
    MlaPlan p;
    plan(ctx_lens, B, p);
    const int nsplit = (int)p.splits.size();
    const size_t need = ws_bytes(nsplit, B, H);
    if (workspace_bytes < need || !workspace)
        return set_error(K3CUDA_ERR_WORKSPACE, "mla_decode: workspace %zu < %zu", workspace_bytes,
                         need);
    K3_ARG_CHECK(aligned(workspace, 256), "workspace must be 256-byte aligned");
    char *w = (char *)workspace;
    SplitDesc *d_splits = (SplitDesc *)w;
    w += align256((size_t)nsplit * sizeof(SplitDesc));
    int *d_slot0 = (int *)w;
    w += align256((size_t)(B + 1) * sizeof(int));
    float *qabs = (float *)w;
    w += align256((size_t)B * H * MLA_QW * sizeof(float));
    float *part = (float *)w;
    K3_CUDA_TRY(cudaMemcpyAsync(d_splits, p.splits.data(), (size_t)nsplit * sizeof(SplitDesc),
                                cudaMemcpyHostToDevice, ctx->stream));
    K3_CUDA_TRY(cudaMemcpyAsync(d_slot0, p.slot0.data(), (size_t)(B + 1) * sizeof(int),
                                cudaMemcpyHostToDevice, ctx->stream));
    const __nv_bfloat16 *qn = (const __nv_bfloat16 *)q_nope, *qr = (const __nv_bfloat16 *)q_rope;
    mla_q_absorb<<<dim3(H, (B + 15) / 16), 256, 0, ctx->stream>>>(
        qn, qr, (const __nv_bfloat16 *)w_uk, qabs, B, H);
    rc = after_launch(ctx, "mla_q_absorb");
    if (rc) return rc;
    const size_t smem = ((size_t)MLA_HG * MLA_QW + MLA_TILE * MLA_QW + MLA_HG * MLA_TILE + 3 * MLA_HG) *
                        sizeof(float);
    K3_CUDA_TRY(cudaFuncSetAttribute(mla_attend_split, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
    mla_attend_split<<<dim3(nsplit, (H + MLA_HG - 1) / MLA_HG), 256, smem, ctx->stream>>>(
        d_splits, qabs, (const __nv_bfloat16 *)latent, (const __nv_bfloat16 *)rope, part, H, cap,
        scale);
    rc = after_launch(ctx, "mla_attend_split");
    if (rc) return rc;
    if (out_dtype == K3CUDA_BF16)
        mla_merge_project<__nv_bfloat16><<<dim3(B, H), 128, 0, ctx->stream>>>(
            part, d_slot0, (const __nv_bfloat16 *)w_uv, (__nv_bfloat16 *)out, H);
    else
        mla_merge_project<float><<<dim3(B, H), 128, 0, ctx->stream>>>(
            part, d_slot0, (const __nv_bfloat16 *)w_uv, (float *)out, H);
    return after_launch(ctx, "mla_merge_project");
}
