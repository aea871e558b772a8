// kda_decode.cu -- KDA single-token recurrent decode on fp32 state (HBM-bound).
//
// Replaces the per-head k3_kda_step call at T = 1 (reference src/core/k3_ops.c:186-243,
// driven by k3_ops.c:927-938). Per stream (sequence, head), with S [dk][dv] row-major:
//     S' = diag(alpha) S                    (k3_ops.c:191-195)
//     u  = S'^T k                           (k3_ops.c:218-223)
//     S''= S' + k (beta (v - u))^T          (k3_ops.c:227-232)
//     o  = S''^T q                          (k3_ops.c:235-241)
// The state is read once and written once: o is formed from the pre-update read as
//     o = S'^T q + (q . k) beta (v - u)
// which is algebraically S''^T q, so no second pass over S is needed.
//
// Fast path (dv == 128, dk in {64,128}): one CTA of 256 threads per stream. Warp w owns
// rows [w*dk/8, (w+1)*dk/8); lane l owns columns [4l, 4l+4). Every thread issues its
// dk/8 128-bit loads of S before anything else, so each SM has up to 2 x 64 KB of state
// reads in flight; the two column reductions (u and S'^T q) cross the 8 warps through
// 8 KB of shared memory; the state goes back with 128-bit streaming stores.
#include <algorithm>

#include "internal.cuh"

namespace k3 {

template <typename IO, int DK>
__global__ void __launch_bounds__(256, 2)
kda_decode_dv128(float *__restrict__ state, IO *__restrict__ o, const IO *__restrict__ q,
                 const IO *__restrict__ k, const IO *__restrict__ v,
                 const float *__restrict__ gate, const float *__restrict__ beta,
                 float q_scale, int gate_is_log) {
    pdl_trigger();
    pdl_wait();  // the state and the inputs may come from the previous kernel
    constexpr int DV = 128;
    constexpr int RPW = DK / 8;  // rows per warp
    const int sh = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    float4 *Sg = reinterpret_cast<float4 *>(state + (size_t)sh * DK * DV);
    float4 s[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++) s[r] = __ldcs(Sg + (size_t)(warp * RPW + r) * (DV / 4) + lane);

    __shared__ float sh_alpha[DK], sh_k[DK], sh_q[DK];
    __shared__ __align__(16) float sh_v[DV];
    __shared__ float4 red_u[8][32], red_w[8][32];
    __shared__ float sh_qk[8];

    float qk_part = 0.f;
    if (tid < DK) {
        const size_t off = (size_t)sh * DK + tid;
        const float gi = gate[off];
        const float kk = io<IO>::ld(k + off);
        const float qq = io<IO>::ld(q + off) * q_scale;
        sh_alpha[tid] = gate_is_log ? expf(gi) : gi;
        sh_k[tid] = kk;
        sh_q[tid] = qq;
        qk_part = qq * kk;
    }
    if (tid >= 128 && tid < 128 + DV) sh_v[tid - 128] = io<IO>::ld(v + (size_t)sh * DV + tid - 128);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) qk_part += __shfl_xor_sync(0xffffffffu, qk_part, off);
    if (lane == 0) sh_qk[warp] = qk_part;
    __syncthreads();

    float4 pu = make_float4(0.f, 0.f, 0.f, 0.f), pw = pu;
#pragma unroll
    for (int r = 0; r < RPW; r++) {
        const int i = warp * RPW + r;
        const float a = sh_alpha[i], ki = sh_k[i], qi = sh_q[i];
        s[r].x *= a; s[r].y *= a; s[r].z *= a; s[r].w *= a;
        pu.x += ki * s[r].x; pu.y += ki * s[r].y; pu.z += ki * s[r].z; pu.w += ki * s[r].w;
        pw.x += qi * s[r].x; pw.y += qi * s[r].y; pw.z += qi * s[r].z; pw.w += qi * s[r].w;
    }
    red_u[warp][lane] = pu;
    red_w[warp][lane] = pw;
    __syncthreads();

    float4 u = red_u[0][lane];
#pragma unroll
    for (int w = 1; w < 8; w++) {
        const float4 t = red_u[w][lane];
        u.x += t.x; u.y += t.y; u.z += t.z; u.w += t.w;
    }
    const float b = beta[sh];
    const float4 vv = reinterpret_cast<const float4 *>(sh_v)[lane];
    float4 d;
    d.x = b * (vv.x - u.x); d.y = b * (vv.y - u.y); d.z = b * (vv.z - u.z); d.w = b * (vv.w - u.w);
#pragma unroll
    for (int r = 0; r < RPW; r++) {
        const float ki = sh_k[warp * RPW + r];
        s[r].x += ki * d.x; s[r].y += ki * d.y; s[r].z += ki * d.z; s[r].w += ki * d.w;
        __stcs(Sg + (size_t)(warp * RPW + r) * (DV / 4) + lane, s[r]);
    }
    if (warp == 0) {
        float qk = 0.f;
#pragma unroll
        for (int w = 0; w < DK / 32; w++) qk += sh_qk[w];
        float4 wq = red_w[0][lane];
#pragma unroll
        for (int w = 1; w < 8; w++) {
            const float4 t = red_w[w][lane];
            wq.x += t.x; wq.y += t.y; wq.z += t.z; wq.w += t.w;
        }
        IO *op = o + (size_t)sh * DV + 4 * lane;
        io<IO>::st(op + 0, wq.x + qk * d.x);
        io<IO>::st(op + 1, wq.y + qk * d.y);
        io<IO>::st(op + 2, wq.z + qk * d.z);
        io<IO>::st(op + 3, wq.w + qk * d.w);
    }
}

// General shapes (dk, dv <= 256, dk*dv <= 32768): the four passes of the reference in
// its order, on a shared-memory copy of one stream's state.
template <typename IO>
__global__ void __launch_bounds__(256)
kda_decode_general(float *__restrict__ state, IO *__restrict__ o, const IO *__restrict__ q,
                   const IO *__restrict__ k, const IO *__restrict__ v,
                   const float *__restrict__ gate, const float *__restrict__ beta, int dk,
                   int dv, float q_scale, int gate_is_log) {
    pdl_trigger();
    pdl_wait();  // the state and the inputs may come from the previous kernel
    extern __shared__ float smem[];
    float *S = smem;                       // [dk][dv]
    float *al = S + (size_t)dk * dv;       // [dk]
    float *kk = al + dk, *qq = kk + dk;    // [dk] each
    float *vv = qq + dk, *u = vv + dv;     // [dv] each
    const int sh = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    float *Sg = state + (size_t)sh * dk * dv;
    for (int i = tid; i < dk; i += nt) {
        const size_t off = (size_t)sh * dk + i;
        const float gi = gate[off];
        al[i] = gate_is_log ? expf(gi) : gi;
        kk[i] = io<IO>::ld(k + off);
        qq[i] = io<IO>::ld(q + off) * q_scale;
    }
    for (int j = tid; j < dv; j += nt) vv[j] = io<IO>::ld(v + (size_t)sh * dv + j);
    __syncthreads();
    for (int e = tid; e < dk * dv; e += nt) S[e] = Sg[e] * al[e / dv];
    __syncthreads();
    for (int j = tid; j < dv; j += nt) {
        float acc = 0.f;
        for (int i = 0; i < dk; i++) acc += kk[i] * S[i * dv + j];
        u[j] = acc;
    }
    __syncthreads();
    const float b = beta[sh];
    for (int e = tid; e < dk * dv; e += nt) {
        const int i = e / dv, j = e - i * dv;
        const float s2 = S[e] + kk[i] * b * (vv[j] - u[j]);
        S[e] = s2;
        Sg[e] = s2;
    }
    __syncthreads();
    for (int j = tid; j < dv; j += nt) {
        float acc = 0.f;
        for (int i = 0; i < dk; i++) acc += qq[i] * S[i * dv + j];
        io<IO>::st(o + (size_t)sh * dv + j, acc);
    }
}

template <typename IO>
static int launch_decode(k3cuda_ctx *ctx, float *state, void *o, const void *q, const void *k,
                         const void *v, const float *gate, const float *beta, int nstream,
                         int dk, int dv, float q_scale, int gate_is_log) {
    const IO *qp = (const IO *)q, *kp = (const IO *)k, *vp = (const IO *)v;
    IO *op = (IO *)o;
    if (dv == 128 && dk == 128 && aligned(state, 16))
        return launch_pdl(ctx, ctx->stream, "kda_decode_dv128<128>", kda_decode_dv128<IO, 128>,
                          dim3(nstream), dim3(256), 0, state, op, qp, kp, vp, gate, beta, q_scale,
                          gate_is_log);
    if (dv == 128 && dk == 64 && aligned(state, 16))
        return launch_pdl(ctx, ctx->stream, "kda_decode_dv128<64>", kda_decode_dv128<IO, 64>,
                          dim3(nstream), dim3(256), 0, state, op, qp, kp, vp, gate, beta, q_scale,
                          gate_is_log);
    const size_t smem = ((size_t)dk * dv + 3 * dk + 2 * dv) * sizeof(float);
    if (smem > 48 * 1024)
        if (int rc_ = set_smem(kda_decode_general<IO>, (int)smem)) return rc_;
    return launch_pdl(ctx, ctx->stream, "kda_decode_general", kda_decode_general<IO>,
                      dim3(nstream), dim3(256), smem, state, op, qp, kp, vp, gate, beta, dk, dv,
                      q_scale, gate_is_log);
}

}  // namespace k3

using namespace k3;

extern "C" int k3cuda_kda_decode(k3cuda_ctx *ctx, float *state, void *o, const void *q,
                                 const void *k, const void *v, const float *gate,
                                 const float *beta, int n_streams, int H, int dk, int dv,
                                 float q_scale, int io_dtype, int gate_mode) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(n_streams >= 0 && H >= 1, "bad n_streams=%d H=%d", n_streams, H);
    K3_ARG_CHECK(io_dtype == K3CUDA_F32 || io_dtype == K3CUDA_BF16, "bad io_dtype %d", io_dtype);
    K3_ARG_CHECK(gate_mode == K3CUDA_GATE_LOG || gate_mode == K3CUDA_GATE_ALPHA,
                 "bad gate_mode %d", gate_mode);
    if (dk < 1 || dv < 1 || dk > 256 || dv > 256 || (size_t)dk * dv > 32768)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "kda_decode: dk=%d dv=%d not built", dk, dv);
    if (n_streams == 0) return K3CUDA_OK;
    K3_ARG_CHECK(state && o && q && k && v && gate && beta, "kda_decode: null pointer");
    const long long ns = (long long)n_streams * H;
    K3_ARG_CHECK(ns <= 0x7fffffffLL, "too many streams");
    const int gl = gate_mode == K3CUDA_GATE_LOG;
    if (io_dtype == K3CUDA_BF16)
        return launch_decode<__nv_bfloat16>(ctx, state, o, q, k, v, gate, beta, (int)ns, dk, dv,
                                            q_scale, gl);
    return launch_decode<float>(ctx, state, o, q, k, v, gate, beta, (int)ns, dk, dv, q_scale, gl);
}

// ------------------------------------------------------------ host-buffer decode step
namespace {
size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// Device staging image of one step: q, k [ns][dk] and v, o [ns][dv] in io dtype, gate
// [ns][dk] and beta [ns] fp32, each region 256-byte aligned.
struct HostStage {
    size_t q, k, v, o, g, b, total;
    HostStage(long long ns, int dk, int dv, size_t es) {
        q = 0;
        k = q + al256((size_t)ns * dk * es);
        v = k + al256((size_t)ns * dk * es);
        o = v + al256((size_t)ns * dv * es);
        g = o + al256((size_t)ns * dv * es);
        b = g + al256((size_t)ns * dk * 4);
        total = b + al256((size_t)ns * 4);
    }
};
}  // namespace

extern "C" int k3cuda_kda_decode_host_workspace(int n_streams, int H, int dk, int dv,
                                                int io_dtype, size_t *bytes) {
    K3_ARG_CHECK(bytes, "null output pointer");
    *bytes = 0;
    K3_ARG_CHECK(n_streams >= 0 && H >= 1 && dk >= 1 && dv >= 1, "bad n_streams=%d H=%d dk=%d dv=%d",
                 n_streams, H, dk, dv);
    K3_ARG_CHECK(io_dtype == K3CUDA_F32 || io_dtype == K3CUDA_BF16, "bad io_dtype %d", io_dtype);
    *bytes = HostStage((long long)n_streams * H, dk, dv, io_dtype == K3CUDA_BF16 ? 2 : 4).total;
    return K3CUDA_OK;
}

extern "C" int k3cuda_kda_decode_host(k3cuda_ctx *ctx, float *state, void *o, const void *q,
                                      const void *k, const void *v, const float *gate,
                                      const float *beta, int n_streams, int H, int dk, int dv,
                                      float q_scale, int io_dtype, int gate_mode, int slices,
                                      void *staging, size_t staging_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(n_streams >= 0 && H >= 1, "bad n_streams=%d H=%d", n_streams, H);
    K3_ARG_CHECK(io_dtype == K3CUDA_F32 || io_dtype == K3CUDA_BF16, "bad io_dtype %d", io_dtype);
    K3_ARG_CHECK(gate_mode == K3CUDA_GATE_LOG || gate_mode == K3CUDA_GATE_ALPHA,
                 "bad gate_mode %d", gate_mode);
    K3_ARG_CHECK(slices >= K3CUDA_HOST_IN_PLACE, "bad slices %d", slices);
    if (dk < 1 || dv < 1 || dk > 256 || dv > 256 || (size_t)dk * dv > 32768)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "kda_decode_host: dk=%d dv=%d not built", dk, dv);
    if (n_streams == 0) return K3CUDA_OK;
    K3_ARG_CHECK(state && o && q && k && v && gate && beta, "kda_decode_host: null pointer");
    const long long ns = (long long)n_streams * H;
    K3_ARG_CHECK(ns <= 0x7fffffffLL, "too many streams");
    const size_t es = io_dtype == K3CUDA_BF16 ? 2 : 4;
    const size_t in_bytes = (size_t)ns * ((2 * (size_t)dk + dv) * es + 4 * (size_t)dk + 4);
    // Measured on the B200 (H = 32, d = 128, bf16): in place costs ~15 us + 2.6 us per
    // sequence (the kernel's PCIe reads are small and latency-bound, ~14 GB/s), the copies
    // ~36 us + 1.35 us per sequence at ~49 GB/s: in place wins below ~17 sequences (~700 KB
    // of inputs); above ~4 MB two slices beat one, and more slices lose to per-copy costs.
    constexpr size_t kInPlaceMax = 640 << 10, kTwoSlices = 4 << 20;
    if (slices == K3CUDA_HOST_IN_PLACE || (slices == 0 && in_bytes <= kInPlaceMax)) {
        // page-locked host memory is mapped into the device's address space: the kernel reads
        // the inputs and writes the output in place over PCIe, with no copy and one launch
        const void *hp[6] = {o, q, k, v, gate, beta};
        void *dp[6];
        bool all = true;
        for (int i = 0; i < 6; i++) {
            cudaPointerAttributes a;
            if (cudaPointerGetAttributes(&a, hp[i]) != cudaSuccess) {
                cudaGetLastError();  // not a CUDA-known pointer: pageable memory
                a.type = cudaMemoryTypeUnregistered;
                a.devicePointer = nullptr;
            }
            dp[i] = a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
            all = all && dp[i];
        }
        if (all)
            return k3cuda_kda_decode(ctx, state, dp[0], dp[1], dp[2], dp[3], (const float *)dp[4],
                                     (const float *)dp[5], n_streams, H, dk, dv, q_scale, io_dtype,
                                     gate_mode);
        K3_ARG_CHECK(slices == 0, "kda_decode_host: in-place mode needs page-locked host buffers");
    }
    K3_ARG_CHECK(staging, "kda_decode_host: null staging buffer");
    const HostStage L(ns, dk, dv, es);
    if (staging_bytes < L.total)
        return set_error(K3CUDA_ERR_WORKSPACE, "kda_decode_host: staging %zu < %zu bytes",
                         staging_bytes, L.total);
    K3_ARG_CHECK(aligned(staging, 256), "kda_decode_host: staging must be 256-byte aligned");
    int S = slices > 0 ? slices : (in_bytes >= kTwoSlices ? 2 : 1);
    S = std::min(S, std::min(n_streams, K3CUDA_HOST_SLICES));
    uint8_t *st = (uint8_t *)staging;
    const uint8_t *hq = (const uint8_t *)q, *hk = (const uint8_t *)k, *hv = (const uint8_t *)v;
    const uint8_t *hg = (const uint8_t *)gate, *hb = (const uint8_t *)beta;
    uint8_t *ho = (uint8_t *)o;
    // A page-locked output is written by the kernels in place: the GPU's writes to host memory
    // are posted and overlap the step, and the device-to-host copies disappear.
    uint8_t *od = nullptr;
    {
        cudaPointerAttributes a;
        const cudaError_t pe = cudaPointerGetAttributes(&a, o);
        if (pe != cudaSuccess)
            cudaGetLastError();  // not a CUDA-known pointer: pageable memory
        else if (a.type == cudaMemoryTypeHost)
            od = (uint8_t *)a.devicePointer;
    }

    K3_CUDA_TRY(cudaEventRecord(ctx->ev_cp_start, ctx->stream));
    K3_CUDA_TRY(cudaStreamWaitEvent(ctx->cp_in, ctx->ev_cp_start, 0));
    K3_CUDA_TRY(cudaStreamWaitEvent(ctx->cp_out, ctx->ev_cp_start, 0));
    cudaError_t e = cudaSuccess;
    for (int s = 0; s < S && rc == K3CUDA_OK && e == cudaSuccess; s++) {
        const long long b0 = (long long)n_streams * s / S, b1 = (long long)n_streams * (s + 1) / S;
        const long long r0 = b0 * H, nr = (b1 - b0) * H;  // (sequence, head) rows of the slice
        if (nr == 0) continue;
        const size_t qo = (size_t)r0 * dk * es, qn = (size_t)nr * dk * es;
        const size_t vo = (size_t)r0 * dv * es, vn = (size_t)nr * dv * es;
        const size_t go = (size_t)r0 * dk * 4, gn = (size_t)nr * dk * 4;
        const cudaMemcpyKind H2D = cudaMemcpyHostToDevice;
        e = cudaMemcpyAsync(st + L.q + qo, hq + qo, qn, H2D, ctx->cp_in);
        if (e == cudaSuccess) e = cudaMemcpyAsync(st + L.k + qo, hk + qo, qn, H2D, ctx->cp_in);
        if (e == cudaSuccess) e = cudaMemcpyAsync(st + L.v + vo, hv + vo, vn, H2D, ctx->cp_in);
        if (e == cudaSuccess) e = cudaMemcpyAsync(st + L.g + go, hg + go, gn, H2D, ctx->cp_in);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(st + L.b + r0 * 4, hb + r0 * 4, (size_t)nr * 4, H2D, ctx->cp_in);
        if (e == cudaSuccess) e = cudaEventRecord(ctx->ev_in[s], ctx->cp_in);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, ctx->ev_in[s], 0);
        if (e != cudaSuccess) break;
        rc = k3cuda_kda_decode(ctx, state + (size_t)r0 * dk * dv, od ? od + vo : st + L.o + vo,
                               st + L.q + qo, st + L.k + qo, st + L.v + vo,
                               (const float *)(st + L.g + go),
                               (const float *)(st + L.b + r0 * 4), (int)(b1 - b0), H, dk, dv,
                               q_scale, io_dtype, gate_mode);
        if (rc) break;
        if (od) continue;  // the output went straight to the host
        e = cudaEventRecord(ctx->ev_k[s], ctx->stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->cp_out, ctx->ev_k[s], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(ho + vo, st + L.o + vo, vn, cudaMemcpyDeviceToHost, ctx->cp_out);
    }
    // both copy streams join the context's stream whatever happened above
    cudaError_t e2 = cudaEventRecord(ctx->ev_cp_in_done, ctx->cp_in);
    if (e2 == cudaSuccess) e2 = cudaStreamWaitEvent(ctx->stream, ctx->ev_cp_in_done, 0);
    cudaError_t e3 = cudaEventRecord(ctx->ev_cp_out_done, ctx->cp_out);
    if (e3 == cudaSuccess) e3 = cudaStreamWaitEvent(ctx->stream, ctx->ev_cp_out_done, 0);
    if (rc) return rc;
    if (e == cudaSuccess) e = e2 != cudaSuccess ? e2 : e3;
    if (e != cudaSuccess)
        return set_error(K3CUDA_ERR_CUDA, "kda_decode_host: %s", cudaGetErrorString(e));
    return K3CUDA_OK;
}
