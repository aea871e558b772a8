// mla_layer.cu -- the MLA layer forward of k3_mla_cached (src/core/k3_ops.c:321-424) with its
// KV cache on the device as the compressed latent (+ the shared rope slot) instead of the
// expanded per-head keys and values.
//
//   step (reference line)                                  here
//   ql = RMSNorm(q_a x) (q_a_norm); q = q_b ql   (:358-360)  projections; rmsnorm_rows
//   ct = kv_a x; RMSNorm(ct[:kv_lora]) (kv_a_norm);           projection; k3cuda_mla_cache_append
//       rope slot ct[kv_lora:] copied unrotated (:363-366)     (writes the latent / rope rows)
//   kv = kv_b ct[:kv_lora] into the cache (:367)             not formed: W_UK, W_UV stay in kv_b
//   causal attention, scale (qk_nope+qk_rope)^-0.5 (:381-411) mla_attend_kvb (absorbed form)
//   acc *= sigmoid(g x) (when g), out = o acc (:413-420)      mla_gate; projection
//
// Projections go through the same streaming / GEMM paths as the KDA layer (kda_layer.cu,
// gemm.cu).
#include "internal.cuh"

namespace k3 {

constexpr int ML_DN = 128, ML_DR = 64, ML_DL = 512, ML_DV = 128;

// y[r] = w * x[r] * inv, inv = 1/sqrt(mean(x^2) + eps) with the sum in double (k3_rmsnorm,
// k3_ops.c:94-101), one row per block, in place. Rows up to RN_CACHE * blockDim elements
// are read once, all loads in flight together, and kept in registers for the scaling.
constexpr int RN_CACHE = 8;
__global__ void rmsnorm_rows(float *__restrict__ x, const float *__restrict__ w, int n,
                             float eps) {
    pdl_trigger();
    pdl_wait();
    __shared__ double red[32];
    float *row = x + (size_t)blockIdx.x * n;
    double ss = 0.0;
    if (n <= RN_CACHE * (int)blockDim.x) {
        float v[RN_CACHE], wv[RN_CACHE];
#pragma unroll
        for (int j = 0; j < RN_CACHE; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            v[j] = i < n ? row[i] : 0.f;
            wv[j] = i < n ? w[i] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < RN_CACHE; j++) ss = fma((double)v[j], (double)v[j], ss);
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x < 32) {
            double t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
#pragma unroll
            for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            if (threadIdx.x == 0) red[0] = t;
        }
        __syncthreads();
        const float inv = (float)(1.0 / sqrt(red[0] / (double)n + (double)eps));
#pragma unroll
        for (int j = 0; j < RN_CACHE; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            if (i < n) row[i] = wv[j] * v[j] * inv;
        }
        return;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fma((double)row[i], (double)row[i], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = (float)(1.0 / sqrt(red[0] / (double)n + (double)eps));
    for (int i = threadIdx.x; i < n; i += blockDim.x) row[i] = w[i] * row[i] * inv;
}

// q [T][H][dn + dr] fp32 -> q_nope [T][H][dn], q_rope [T][H][dr] bf16 (grid-stride over
// all T*H*(dn+dr) elements)
__global__ void mla_q_split(__nv_bfloat16 *__restrict__ qn, __nv_bfloat16 *__restrict__ qr,
                            const float *__restrict__ q, long long n) {
    pdl_trigger();
    pdl_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long th = i / (ML_DN + ML_DR);  // (token, head) row
        const int c = (int)(i - th * (ML_DN + ML_DR));
        const __nv_bfloat16 v = __float2bfloat16_rn(q[i]);
        if (c < ML_DN) qn[th * ML_DN + c] = v;
        else qr[th * ML_DR + c - ML_DN] = v;
    }
}

__global__ void f32_to_bf16(__nv_bfloat16 *__restrict__ y, const float *__restrict__ x,
                            long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        y[i] = __float2bfloat16_rn(x[i]);
}

// ot = acc * sigmoid(g x) (or acc when there is no gate), also as the bf16 hi/lo split when
// o_proj is a bf16 GEMM
__global__ void mla_gate(float *__restrict__ ot, __nv_bfloat16 *__restrict__ hi,
                         __nv_bfloat16 *__restrict__ lo, const float *__restrict__ acc,
                         const float *__restrict__ gb, long long n) {
    pdl_trigger();  // o_proj's CTAs may be scheduled while this kernel runs
    pdl_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v = acc[i];
        if (gb) v *= 1.0f / (1.0f + expf(-gb[i]));
        ot[i] = v;
        if (hi) {
            const __nv_bfloat16 h = __float2bfloat16_rn(v);
            hi[i] = h;
            lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
        }
    }
}

static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

struct MlaLayerPlan {
    size_t ql, ct, gb, q, qn, qr, acc, ot, xs, qls, ots, kvb, att, total;
    bool gemm, split;
};

static void plan(int T, int E, int H, int q_lora, int cached, int wdt, MlaLayerPlan *p) {
    size_t off = 0;
    auto take = [&](size_t b) { const size_t o = off; off += al256(b); return o; };
    const size_t HV = (size_t)H * ML_DV, HQ = (size_t)H * (ML_DN + ML_DR);
    p->gemm = T > PROJ_MAXT;
    p->split = p->gemm && wdt == K3CUDA_BF16;
    p->ql = take((size_t)T * q_lora * 4);
    p->ct = take((size_t)T * (ML_DL + ML_DR) * 4);
    p->gb = take((size_t)T * HV * 4);
    p->q = take((size_t)T * HQ * 4);
    p->qn = take((size_t)T * H * ML_DN * 2);
    p->qr = take((size_t)T * H * ML_DR * 2);
    p->acc = take((size_t)T * HV * 4);
    p->ot = take((size_t)T * HV * 4);
    p->xs = p->split ? take((size_t)2 * T * E * 2) : 0;
    p->qls = p->split ? take((size_t)2 * T * q_lora * 2) : 0;
    p->ots = p->split ? take((size_t)2 * T * HV * 2) : 0;
    p->kvb = wdt == K3CUDA_F32 ? take((size_t)H * (ML_DN + ML_DV) * ML_DL * 2) : 0;
    p->att = take(mla_attend_kvb_workspace(T, cached, H));
    p->total = off;
}

static int shape_ok(int T, int E, int H, int q_lora, int dn, int dr, int dl, int dv, int wdt,
                    int cached, int cap) {
    K3_ARG_CHECK(T >= 0 && E >= 8 && H >= 1 && q_lora >= 8 && cached >= 0 && cap >= 1,
                 "mla_layer: bad shape T=%d E=%d H=%d q_lora=%d cached=%d cap=%d", T, E, H,
                 q_lora, cached, cap);
    K3_ARG_CHECK(wdt == K3CUDA_F32 || wdt == K3CUDA_BF16, "mla_layer: bad wdt %d", wdt);
    if (dn != ML_DN || dr != ML_DR || dl != ML_DL || dv != ML_DV || H > 128 || E % 8 ||
        q_lora % 8)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "mla_layer: dn=%d dr=%d dl=%d dv=%d H=%d E=%d "
                         "q_lora=%d not built (the released head geometry 128/64/512/128, "
                         "H <= 128, E and q_lora multiples of 8)", dn, dr, dl, dv, H, E, q_lora);
    if ((long long)cached + T > cap)
        return set_error(K3CUDA_ERR_ARG, "mla_layer: position %lld past the cache (cap %d)",
                         (long long)cached + T - 1, cap);
    return K3CUDA_OK;
}

static int grid_for(k3cuda_ctx *ctx, long long n) {
    const long long want = (n + 255) / 256;
    return (int)(want < 8LL * ctx->sm_count ? (want > 0 ? want : 1) : 8LL * ctx->sm_count);
}

}  // namespace k3

using namespace k3;

extern "C" int k3cuda_mla_layer_workspace(int T, int E, int H, int q_lora, int cached, int wdt,
                                          size_t *bytes) {
    K3_ARG_CHECK(bytes, "null bytes");
    int rc = shape_ok(T, E, H, q_lora, ML_DN, ML_DR, ML_DL, ML_DV, wdt, cached, cached + T);
    if (rc) return rc;
    MlaLayerPlan p;
    plan(T, E, H, q_lora, cached, wdt, &p);
    *bytes = p.total;
    return K3CUDA_OK;
}

extern "C" int k3cuda_mla_layer(k3cuda_ctx *ctx, float *out, const float *x,
                                const k3cuda_mla_weights *w, int T, int E, int H, int q_lora,
                                int dn, int dr, int dl, int dv, float rms_eps, void *latent,
                                void *rope, int cached, int cap, void *workspace,
                                size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(w, "mla_layer: null weights");
    if ((rc = shape_ok(T, E, H, q_lora, dn, dr, dl, dv, w->wdt, cached, cap))) return rc;
    if (T == 0) return K3CUDA_OK;
    K3_ARG_CHECK(out && x && w->q_a && w->q_b && w->kv_a && w->kv_b && w->o && w->q_a_norm &&
                 w->kv_a_norm && latent && rope, "mla_layer: null pointer");
    const void *al[] = {out, x, w->q_a, w->q_b, w->kv_a, w->kv_b, w->o, w->q_a_norm,
                        w->kv_a_norm, latent, rope};
    for (const void *p : al)
        K3_ARG_CHECK(aligned(p, 16), "mla_layer: pointers must be 16-byte aligned");
    K3_ARG_CHECK(!w->g || aligned(w->g, 16), "mla_layer: g must be 16-byte aligned");
    MlaLayerPlan pl;
    plan(T, E, H, q_lora, cached, w->wdt, &pl);
    if (workspace_bytes < pl.total || !workspace)
        return set_error(K3CUDA_ERR_WORKSPACE, "mla_layer: workspace %zu < %zu bytes",
                         workspace_bytes, pl.total);
    K3_ARG_CHECK(aligned(workspace, 256), "mla_layer: workspace must be 256-byte aligned");
    char *ws = (char *)workspace;
    const int wdt = w->wdt, HV = H * ML_DV, HQ = H * (ML_DN + ML_DR), KW = ML_DL + ML_DR;
    float *ql = (float *)(ws + pl.ql), *ct = (float *)(ws + pl.ct), *gb = (float *)(ws + pl.gb);
    float *q = (float *)(ws + pl.q), *acc = (float *)(ws + pl.acc), *ot = (float *)(ws + pl.ot);
    __nv_bfloat16 *qn = (__nv_bfloat16 *)(ws + pl.qn), *qr = (__nv_bfloat16 *)(ws + pl.qr);
    __nv_bfloat16 *xs = pl.split ? (__nv_bfloat16 *)(ws + pl.xs) : nullptr;
    __nv_bfloat16 *qls = pl.split ? (__nv_bfloat16 *)(ws + pl.qls) : nullptr;
    __nv_bfloat16 *ots = pl.split ? (__nv_bfloat16 *)(ws + pl.ots) : nullptr;
    // projections of x: q_a, kv_a and the gate
    bool forked = false;
    if (!pl.gemm) {
        Proj pr[2] = {{w->q_a, ql, q_lora}, {w->kv_a, ct, KW}};
        if ((rc = matvec(ctx, x, T, E, pr, 2, wdt))) return rc;
        if (w->g) {
            // the gate projection (needed only at the gate) streams on the side stream while
            // the chain of small, latency-bound steps up to the attention runs on the main one
            K3_CUDA_TRY(cudaEventRecord(ctx->ev_fork, ctx->stream));
            K3_CUDA_TRY(cudaStreamWaitEvent(ctx->aux, ctx->ev_fork, 0));
            cudaStream_t main_stream = ctx->stream;
            ctx->stream = ctx->aux;
            const Proj gate{w->g, gb, HV};
            rc = matvec(ctx, x, T, E, &gate, 1, wdt);
            ctx->stream = main_stream;
            if (rc) return rc;
            K3_CUDA_TRY(cudaEventRecord(ctx->ev_join, ctx->aux));
            forked = true;
        }
    } else {
        if (pl.split && (rc = split(ctx, xs, x, (long long)T * E))) return rc;
        if ((rc = gemm(ctx, ql, x, xs, w->q_a, wdt, T, E, q_lora))) return rc;
        if ((rc = gemm(ctx, ct, x, xs, w->kv_a, wdt, T, E, KW))) return rc;
        if (w->g && (rc = gemm(ctx, gb, x, xs, w->g, wdt, T, E, HV))) return rc;
    }
    // q = q_b(RMSNorm(ql))
    if ((rc = launch_pdl(ctx, ctx->stream, "rmsnorm_rows", rmsnorm_rows, dim3(T), dim3(256), 0,
                         ql, (const float *)w->q_a_norm, q_lora, rms_eps)))
        return rc;
    if (pl.split && (rc = split(ctx, qls, ql, (long long)T * q_lora))) return rc;
    if ((rc = project(ctx, q, ql, qls, w->q_b, wdt, T, q_lora, HQ))) return rc;
    // the new latent / rope rows (kv_a_norm over the latent only)
    if ((rc = k3cuda_mla_cache_append(ctx, latent, rope, ct, w->kv_a_norm, rms_eps, 0, cached, T,
                                      1, cap, ML_DL, ML_DR)))
        return rc;
    {
        const long long n = (long long)T * HQ;
        if ((rc = launch_pdl(ctx, ctx->stream, "mla_q_split", mla_q_split, dim3(grid_for(ctx, n)),
                             dim3(256), 0, qn, qr, (const float *)q, n)))
            return rc;
    }
    const void *kvb = w->kv_b;
    if (wdt == K3CUDA_F32) {
        const long long n = (long long)H * (ML_DN + ML_DV) * ML_DL;
        f32_to_bf16<<<grid_for(ctx, n), 256, 0, ctx->stream>>>((__nv_bfloat16 *)(ws + pl.kvb),
                                                              (const float *)w->kv_b, n);
        if ((rc = after_launch(ctx, "f32_to_bf16"))) return rc;
        kvb = ws + pl.kvb;
    }
    const float scale = 1.0f / sqrtf((float)(ML_DN + ML_DR));
    if ((rc = mla_attend_kvb(ctx, acc, qn, qr, latent, rope, kvb, T, cached, cap, H, scale,
                             ws + pl.att, pl.total - pl.att)))
        return rc;
    const long long n = (long long)T * HV;
    if (forked) K3_CUDA_TRY(cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
    mla_gate<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(ot, ots, ots ? ots + n : nullptr, acc,
                                                       w->g ? gb : nullptr, n);
    if ((rc = after_launch(ctx, "mla_gate"))) return rc;
    return project(ctx, out, ot, ots, w->o, wdt, T, HV, E);
}

// ---------------------------------------------------------- any head geometry, fp32 cache
// k3_mla_cached for head widths other than the released 128/64/512/128 (the reference's
// own test models use 24/8/32/16): the cache is fp32 latent + rope rows, the attention is
// the absorbed form on CUDA cores with fp32 arithmetic throughout, so the layer stays
// within fp32 rounding of the reference rather than inside a bf16 bound.
namespace k3 {

constexpr int MG_WARPS = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// latent[pos0 + t] = kv_a_norm * ct[t][0:dl] / sqrt(mean(ct[t][0:dl]^2) + eps) (sum of squares
// in double, as k3_rmsnorm) and rope[pos0 + t] = ct[t][dl:dl+dr] (k3_ops.c:363-366); one
// block per token
__global__ void mla_append_f32(float *__restrict__ latent, float *__restrict__ rope,
                               const float *__restrict__ ct, const float *__restrict__ wn,
                               int dl, int dr, int pos0, float eps) {
    __shared__ double red[32];
    const int t = blockIdx.x;
    const float *c = ct + (size_t)t * (dl + dr);
    double ss = 0.0;
    for (int i = threadIdx.x; i < dl; i += blockDim.x) ss = fma((double)c[i], (double)c[i], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = (float)(1.0 / sqrt(red[0] / (double)dl + (double)eps));
    float *lr = latent + (size_t)(pos0 + t) * dl;
    float *rr = rope + (size_t)(pos0 + t) * dr;
    for (int i = threadIdx.x; i < dl; i += blockDim.x) lr[i] = wn[i] * c[i] * inv;
    for (int i = threadIdx.x; i < dr; i += blockDim.x) rr[i] = c[dl + i];
}

// acc[t][h][0:dv] for query t at position cached + t and head h (block (t, h), 8 warps):
//   qa = W_UK[h]^T q_nope                      (W_UK[h] = kv_b rows h*(dn+dv) .. +dn)
//   score[s] = (qa . latent[s] + q_rope . rope[s]) * scale,   s = 0 .. cached + t
//   o_lat = sum_s softmax(score)[s] latent[s];  acc = W_UV[h] o_lat  (the next dv rows)
// the attention of k3_ops.c:381-411 with kv_b's per-head blocks factored through the latent
// (a warp walks every 8th position with its own running max / sum / o_lat, and the warps
// merge at the end). Dynamic shared memory: (dl + dr + 8 dl + 16) floats.
template <typename WT>
__global__ void mla_attend_f32(float *__restrict__ acc, const float *__restrict__ q,
                               const WT *__restrict__ kv_b, const float *__restrict__ latent,
                               const float *__restrict__ rope, int H, int dn, int dr, int dl,
                               int dv, int cached, float scale) {
    extern __shared__ float sm[];
    const int t = blockIdx.x, h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *qa = sm, *qrs = qa + dl, *ow = qrs + dr, *mw = ow + MG_WARPS * dl;
    const float *qt = q + ((size_t)t * H + h) * (dn + dr);
    const WT *wuk = kv_b + (size_t)h * (dn + dv) * dl;
    const WT *wuv = wuk + (size_t)dn * dl;
    for (int j = threadIdx.x; j < dl; j += blockDim.x) {
        float s = 0.f;
        for (int i = 0; i < dn; i++) s = fmaf(qt[i], io<WT>::ld(wuk + (size_t)i * dl + j), s);
        qa[j] = s;
    }
    for (int i = threadIdx.x; i < dr; i += blockDim.x) qrs[i] = qt[dn + i];
    for (int i = threadIdx.x; i < MG_WARPS * dl; i += blockDim.x) ow[i] = 0.f;
    __syncthreads();
    const int P = cached + t + 1;
    float m = -INFINITY, l = 0.f;
    float *o = ow + warp * dl;
    for (int s = warp; s < P; s += MG_WARPS) {
        const float *ls = latent + (size_t)s * dl;
        const float *rs = rope + (size_t)s * dr;
        float d = 0.f;
        for (int i = lane; i < dl; i += 32) d = fmaf(qa[i], ls[i], d);
        for (int i = lane; i < dr; i += 32) d = fmaf(qrs[i], rs[i], d);
        d = warp_sum(d) * scale;
        const float mn = fmaxf(m, d);
        const float corr = expf(m - mn), p = expf(d - mn);
        l = l * corr + p;
        for (int i = lane; i < dl; i += 32) o[i] = fmaf(o[i], corr, p * ls[i]);
        m = mn;
    }
    if (lane == 0) {
        mw[2 * warp] = m;
        mw[2 * warp + 1] = l;
    }
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < MG_WARPS; w++)
        if (mw[2 * w + 1] > 0.f) M = fmaxf(M, mw[2 * w]);
    float L = 0.f;
    for (int w = 0; w < MG_WARPS; w++)
        if (mw[2 * w + 1] > 0.f) L += mw[2 * w + 1] * expf(mw[2 * w] - M);
    const float invL = 1.0f / L;
    for (int i = threadIdx.x; i < dl; i += blockDim.x) {
        float v = 0.f;
        for (int w = 0; w < MG_WARPS; w++)
            if (mw[2 * w + 1] > 0.f) v = fmaf(ow[w * dl + i], expf(mw[2 * w] - M), v);
        qa[i] = v * invL;  // o_lat (qa is no longer needed)
    }
    __syncthreads();
    for (int j = warp; j < dv; j += MG_WARPS) {
        float s = 0.f;
        for (int i = lane; i < dl; i += 32) s = fmaf(io<WT>::ld(wuv + (size_t)j * dl + i), qa[i], s);
        s = warp_sum(s);
        if (lane == 0) acc[((size_t)t * H + h) * dv + j] = s;
    }
}

struct MlaF32Plan {
    size_t ql, ct, gb, q, acc, ot, xs, qls, ots, total;
    bool split;
};

static void plan_f32(int T, int E, int H, int q_lora, int dn, int dr, int dl, int dv, int wdt,
                     MlaF32Plan *p) {
    size_t off = 0;
    auto take = [&](size_t b) { const size_t o = off; off += al256(b); return o; };
    const size_t HV = (size_t)H * dv, HQ = (size_t)H * (dn + dr);
    p->split = T > PROJ_MAXT && wdt == K3CUDA_BF16;
    p->ql = take((size_t)T * q_lora * 4);
    p->ct = take((size_t)T * (dl + dr) * 4);
    p->gb = take((size_t)T * HV * 4);
    p->q = take((size_t)T * HQ * 4);
    p->acc = take((size_t)T * HV * 4);
    p->ot = take((size_t)T * HV * 4);
    p->xs = p->split ? take((size_t)2 * T * E * 2) : 0;
    p->qls = p->split ? take((size_t)2 * T * q_lora * 2) : 0;
    p->ots = p->split ? take((size_t)2 * T * HV * 2) : 0;
    p->total = off;
}

static int shape_f32_ok(int T, int E, int H, int q_lora, int dn, int dr, int dl, int dv, int wdt,
                        int cached, int cap) {
    K3_ARG_CHECK(T >= 0 && H >= 1 && dn >= 1 && dr >= 0 && dv >= 1 && cached >= 0 && cap >= 1,
                 "mla_layer_f32: bad shape T=%d H=%d dn=%d dr=%d dv=%d cached=%d cap=%d", T, H,
                 dn, dr, dv, cached, cap);
    K3_ARG_CHECK(wdt == K3CUDA_F32 || wdt == K3CUDA_BF16, "mla_layer_f32: bad wdt %d", wdt);
    if (E < 8 || E % 8 || q_lora < 8 || q_lora % 8 || (H * dv) % 8 || dl < 1 || dl > 1024 ||
        dr > 256)
        return set_error(K3CUDA_ERR_UNSUPPORTED,
                         "mla_layer_f32: E=%d q_lora=%d H*dv=%d (multiples of 8), dl=%d "
                         "(<= 1024), dr=%d (<= 256) not supported", E, q_lora, H * dv, dl, dr);
    if ((long long)cached + T > cap)
        return set_error(K3CUDA_ERR_ARG, "mla_layer_f32: position %lld past the cache (cap %d)",
                         (long long)cached + T - 1, cap);
    return K3CUDA_OK;
}

}  // namespace k3

extern "C" int k3cuda_mla_layer_f32_workspace(int T, int E, int H, int q_lora, int dn, int dr,
                                              int dl, int dv, int wdt, size_t *bytes) {
    K3_ARG_CHECK(bytes, "null bytes");
    int rc = shape_f32_ok(T, E, H, q_lora, dn, dr, dl, dv, wdt, 0, T > 0 ? T : 1);
    if (rc) return rc;
    MlaF32Plan p;
    plan_f32(T, E, H, q_lora, dn, dr, dl, dv, wdt, &p);
    *bytes = p.total;
    return K3CUDA_OK;
}

extern "C" int k3cuda_mla_layer_f32(k3cuda_ctx *ctx, float *out, const float *x,
                                    const k3cuda_mla_weights *w, int T, int E, int H, int q_lora,
                                    int dn, int dr, int dl, int dv, float rms_eps, float *latent,
                                    float *rope, int cached, int cap, void *workspace,
                                    size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(w, "mla_layer_f32: null weights");
    if ((rc = shape_f32_ok(T, E, H, q_lora, dn, dr, dl, dv, w->wdt, cached, cap))) return rc;
    if (T == 0) return K3CUDA_OK;
    K3_ARG_CHECK(out && x && w->q_a && w->q_b && w->kv_a && w->kv_b && w->o && w->q_a_norm &&
                 w->kv_a_norm && latent && (rope || dr == 0), "mla_layer_f32: null pointer");
    const void *al[] = {out, x, w->q_a, w->q_b, w->kv_a, w->o};
    for (const void *p : al)
        K3_ARG_CHECK(aligned(p, 16), "mla_layer_f32: x, out and the projections must be 16-byte "
                                     "aligned");
    K3_ARG_CHECK(!w->g || aligned(w->g, 16), "mla_layer_f32: g must be 16-byte aligned");
    MlaF32Plan pl;
    plan_f32(T, E, H, q_lora, dn, dr, dl, dv, w->wdt, &pl);
    if (workspace_bytes < pl.total || !workspace)
        return set_error(K3CUDA_ERR_WORKSPACE, "mla_layer_f32: workspace %zu < %zu bytes",
                         workspace_bytes, pl.total);
    K3_ARG_CHECK(aligned(workspace, 256), "mla_layer_f32: workspace must be 256-byte aligned");
    char *ws = (char *)workspace;
    const int wdt = w->wdt, HV = H * dv, HQ = H * (dn + dr);
    float *ql = (float *)(ws + pl.ql), *ct = (float *)(ws + pl.ct), *gb = (float *)(ws + pl.gb);
    float *q = (float *)(ws + pl.q), *acc = (float *)(ws + pl.acc), *ot = (float *)(ws + pl.ot);
    __nv_bfloat16 *xs = pl.split ? (__nv_bfloat16 *)(ws + pl.xs) : nullptr;
    __nv_bfloat16 *qls = pl.split ? (__nv_bfloat16 *)(ws + pl.qls) : nullptr;
    __nv_bfloat16 *ots = pl.split ? (__nv_bfloat16 *)(ws + pl.ots) : nullptr;
    if (pl.split && (rc = split(ctx, xs, x, (long long)T * E))) return rc;
    if ((rc = project(ctx, ql, x, xs, w->q_a, wdt, T, E, q_lora))) return rc;
    if ((rc = project(ctx, ct, x, xs, w->kv_a, wdt, T, E, dl + dr))) return rc;
    if (w->g && (rc = project(ctx, gb, x, xs, w->g, wdt, T, E, HV))) return rc;
    rmsnorm_rows<<<T, 256, 0, ctx->stream>>>(ql, w->q_a_norm, q_lora, rms_eps);
    if ((rc = after_launch(ctx, "rmsnorm_rows"))) return rc;
    if (pl.split && (rc = split(ctx, qls, ql, (long long)T * q_lora))) return rc;
    if ((rc = project(ctx, q, ql, qls, w->q_b, wdt, T, q_lora, HQ))) return rc;
    mla_append_f32<<<T, 256, 0, ctx->stream>>>(latent, rope, ct, w->kv_a_norm, dl, dr, cached,
                                                rms_eps);
    if ((rc = after_launch(ctx, "mla_append_f32"))) return rc;
    const float scale = 1.0f / sqrtf((float)(dn + dr));
    const int smem = (int)((size_t)(dl + dr + MG_WARPS * dl + 2 * MG_WARPS) * sizeof(float));
    if (wdt == K3CUDA_BF16) {
        if ((rc = set_smem(mla_attend_f32<__nv_bfloat16>, smem))) return rc;
        mla_attend_f32<__nv_bfloat16><<<dim3(T, H), 32 * MG_WARPS, smem, ctx->stream>>>(
            acc, q, (const __nv_bfloat16 *)w->kv_b, latent, rope, H, dn, dr, dl, dv, cached,
            scale);
    } else {
        if ((rc = set_smem(mla_attend_f32<float>, smem))) return rc;
        mla_attend_f32<float><<<dim3(T, H), 32 * MG_WARPS, smem, ctx->stream>>>(
            acc, q, (const float *)w->kv_b, latent, rope, H, dn, dr, dl, dv, cached, scale);
    }
    if ((rc = after_launch(ctx, "mla_attend_f32"))) return rc;
    const long long n = (long long)T * HV;
    mla_gate<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(ot, ots, ots ? ots + n : nullptr, acc,
                                                       w->g ? gb : nullptr, n);
    if ((rc = after_launch(ctx, "mla_gate"))) return rc;
    return project(ctx, out, ot, ots, w->o, wdt, T, HV, E);
}
