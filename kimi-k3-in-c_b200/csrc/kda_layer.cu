// kda_layer.cu -- the KDA layer forward of k3_kda_layer (src/core/k3_ops.c:864-951) with
// every activation resident on the device, and the projection primitive k3cuda_matmul
// (k3_mmw, include/k3/k3.h:290-296) it is built from.
//
//   step (reference line)                         where it runs here
//   1   q, k, v, b, f_a, f_b projections (:877-886)  matvec_rows (T <= 8) or gemm (T > 8)
//   2   ShortConv + SiLU, history carried (:889-892)  kda_layer_pre, one launch for
//   3   L2 on q and k per head, eps 1e-6 (:895-899)   steps 2-5
//   4/5 beta = sigmoid, decay chain (:902-906)
//   6   recurrence, q * D^-0.5 (:908-938)           k3cuda_kda_decode / k3cuda_kda_prefill
//   7/8 head RMSNorm, then * sigmoid(g x) (:941-947) kda_layer_post (g x is formed in step 1)
//   9   o_proj (:948)                               matvec_rows or gemm
//
// Projections. Activations are fp32 as in the reference, weights fp32 or bf16 (the wdt tag).
// With T <= 8 tokens every weight is used at most 8 times, so a projection is weight
// streaming: matvec_rows reads each weight row once with 16-byte streaming loads and forms
// the T dot products from exact fp32 products summed in fp32, bound by HBM. The first
// projections of the layer (q, k, v, g, b, f_a all read the same x) go out as ONE launch
// over a table of weight matrices. With T > 8 a projection is a GEMM (gemm.cu): bf16
// weights on tcgen05 with the fp32 activations split into bf16 hi + lo halves (x = hi + lo
// to 2^-16 relative) whose products accumulate into one fp32 tile, so x is not rounded to
// bf16; fp32 weights on the CUDA cores.
#include "internal.cuh"

namespace k3 {

// sigmoid with the fast exponential and the hardware reciprocal (rcp.approx, no slow
// path): within a few ulp of 1 / (1 + expf(-x)) (the reference's sigmoidf_), and exactly 0
// where exp(-x) overflows
__device__ __forceinline__ float dsigm(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + __expf(-x)));
    return r;
}

// ------------------------------------------------------------------- matvec_rows
// y_s[t][r] = sum_i W_s[r][i] x[t][i] for up to MV_MAXSEG weight matrices W_s that share x
// and `in`. A warp owns MV_ROWS rows and one of `ks` slices of `in`; its lanes read 16-byte
// pieces (8 weights) of every row, so a warp load is 512 contiguous bytes per row. The `ks`
// slices of a row group are summed through shared memory in a fixed order.
constexpr int MV_THREADS = 256, MV_WARPS = 8, MV_MAXT = 8, MV_MAXSEG = 8;
// rows per warp: 2 for one token (more warps in flight), 4 for more tokens (each x load
// feeds more rows)
template <int NT> constexpr int mv_rows() { return NT == 1 ? 2 : 4; }

struct MatvecSeg {
    const void *W;  // [rows][in]
    float *y;       // [T][rows]
    int rows;
    int blocks;
};
struct MatvecArgs {
    MatvecSeg seg[MV_MAXSEG];
    int nseg;
    const float *x;  // [T][in]
    int in;
    int ks;
};

// weights are read once per call: no L1 allocation, 256-byte L2 sectors
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float w[8]) {
    const uint4 u = ld_stream(p);
    const unsigned int q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        w[2 * j] = __uint_as_float(q[j] << 16);
        w[2 * j + 1] = __uint_as_float(q[j] & 0xffff0000u);
    }
}
__device__ __forceinline__ void load8(const float *p, float w[8]) {
    const uint4 a = ld_stream(p), b = ld_stream(p + 4);
    w[0] = __uint_as_float(a.x); w[1] = __uint_as_float(a.y);
    w[2] = __uint_as_float(a.z); w[3] = __uint_as_float(a.w);
    w[4] = __uint_as_float(b.x); w[5] = __uint_as_float(b.y);
    w[6] = __uint_as_float(b.z); w[7] = __uint_as_float(b.w);
}

// Raw image of one 8-weight piece (one 16-byte load for bf16, two for fp32), so that pieces
// can be fetched before the kernel waits for its input and unpacked afterwards.
template <typename WT> struct Piece { uint4 u[sizeof(WT) / 2]; };
template <typename WT>
__device__ __forceinline__ void ld_piece(const WT *p, Piece<WT> &q) {
#pragma unroll
    for (int i = 0; i < (int)(sizeof(WT) / 2); i++) q.u[i] = ld_stream(reinterpret_cast<const uint4 *>(p) + i);
}
__device__ __forceinline__ void unpack(const Piece<__nv_bfloat16> &q, float w[8]) {
    const unsigned int v[4] = {q.u[0].x, q.u[0].y, q.u[0].z, q.u[0].w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        w[2 * j] = __uint_as_float(v[j] << 16);
        w[2 * j + 1] = __uint_as_float(v[j] & 0xffff0000u);
    }
}
__device__ __forceinline__ void unpack(const Piece<float> &q, float w[8]) {
    w[0] = __uint_as_float(q.u[0].x); w[1] = __uint_as_float(q.u[0].y);
    w[2] = __uint_as_float(q.u[0].z); w[3] = __uint_as_float(q.u[0].w);
    w[4] = __uint_as_float(q.u[1].x); w[5] = __uint_as_float(q.u[1].y);
    w[6] = __uint_as_float(q.u[1].z); w[7] = __uint_as_float(q.u[1].w);
}

// One-token bf16 streaming is held to 40 registers so that six blocks fit on an SM (measured:
// 6 % faster per MLA layer call than five blocks with the weight prefetch's extra registers).
template <int NT, typename WT>
__global__ void __launch_bounds__(MV_THREADS, (NT == 1 && sizeof(WT) == 2) ? 6 : 1)
matvec_rows(const __grid_constant__ MatvecArgs a) {
    constexpr int MV_ROWS = mv_rows<NT>();
    __shared__ float part[MV_WARPS][MV_ROWS * NT];
    pdl_trigger();
    int b = blockIdx.x, s = 0;
    while (s + 1 < a.nseg && b >= a.seg[s].blocks) b -= a.seg[s++].blocks;
    const MatvecSeg &sg = a.seg[s];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = a.ks, rg = warp / ks, sl = warp - rg * ks;
    const int row0 = (b * (MV_WARPS / ks) + rg) * MV_ROWS;
    const int n8 = a.in >> 3, per = (n8 + ks - 1) / ks;
    const int b8 = sl * per, e8 = min(n8, b8 + per);
    const WT *wr[MV_ROWS];
#pragma unroll
    for (int r = 0; r < MV_ROWS; r++)  // rows past the end re-read the last row, never stored
        wr[r] = (const WT *)sg.W + (size_t)min(row0 + r, sg.rows - 1) * a.in;
    float acc[MV_ROWS][NT];
#pragma unroll
    for (int r = 0; r < MV_ROWS; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[r][t] = 0.f;
    auto step = [&](int i8, const float (&w)[MV_ROWS][8]) {
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float4 *xp = reinterpret_cast<const float4 *>(a.x + (size_t)t * a.in) + 2 * i8;
            const float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
            const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int r = 0; r < MV_ROWS; r++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[r][t] = fmaf(w[r][j], xv[j], acc[r][t]);
        }
    };
    // The first MV_PF pieces of every row are in flight before the wait: the weights never
    // depend on the previous kernel, so their fetch overlaps its tail.
    constexpr int MV_PF = 2;
    Piece<WT> pre[MV_PF][MV_ROWS];
#pragma unroll
    for (int u = 0; u < MV_PF; u++) {
        const int i8 = b8 + lane + 32 * u;
#pragma unroll
        for (int r = 0; r < MV_ROWS; r++)
            if (i8 < e8) ld_piece(wr[r] + (size_t)i8 * 8, pre[u][r]);
    }
    pdl_wait();  // x comes from the previous kernel
#pragma unroll
    for (int u = 0; u < MV_PF; u++) {
        const int i8 = b8 + lane + 32 * u;
        if (i8 < e8) {
            float w[MV_ROWS][8];
#pragma unroll
            for (int r = 0; r < MV_ROWS; r++) unpack(pre[u][r], w[r]);
            step(i8, w);
        }
    }
#pragma unroll 2
    for (int i8 = b8 + lane + 32 * MV_PF; i8 < e8; i8 += 32) {
        float w[MV_ROWS][8];
#pragma unroll
        for (int r = 0; r < MV_ROWS; r++) load8(wr[r] + (size_t)i8 * 8, w[r]);
        step(i8, w);
    }
#pragma unroll
    for (int r = 0; r < MV_ROWS; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) {
            float v = acc[r][t];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) part[warp][r * NT + t] = v;
        }
    __syncthreads();
    if (sl == 0 && lane < MV_ROWS * NT) {
        const int r = lane / NT, t = lane - r * NT;
        float v = 0.f;
        for (int j = 0; j < ks; j++) v += part[rg * ks + j][lane];
        if (row0 + r < sg.rows) sg.y[(size_t)t * sg.rows + row0 + r] = v;
    }
}

// On the context's stream the launch overlaps the previous kernel's tail (PDL); on the side
// stream, whose work is ordered by events, it is a plain launch.
template <int NT>
static int launch_matvec(k3cuda_ctx *ctx, const MatvecArgs &a, int wdt, int blocks) {
    if (ctx->stream == ctx->aux) {
        if (wdt == K3CUDA_BF16)
            matvec_rows<NT, __nv_bfloat16><<<blocks, MV_THREADS, 0, ctx->stream>>>(a);
        else
            matvec_rows<NT, float><<<blocks, MV_THREADS, 0, ctx->stream>>>(a);
        return after_launch(ctx, "matvec_rows");
    }
    if (wdt == K3CUDA_BF16)
        return launch_pdl(ctx, ctx->stream, "matvec_rows", matvec_rows<NT, __nv_bfloat16>,
                          dim3(blocks), dim3(MV_THREADS), 0, a);
    return launch_pdl(ctx, ctx->stream, "matvec_rows", matvec_rows<NT, float>, dim3(blocks),
                      dim3(MV_THREADS), 0, a);
}

// One launch of matvec_rows over `n` projections of the same x [T][in] (T <= MV_MAXT).
int matvec(k3cuda_ctx *ctx, const float *x, int T, int in, const Proj *p, int n, int wdt) {
    if (T < 1 || T > MV_MAXT || n < 1 || n > MV_MAXSEG)
        return set_error(K3CUDA_ERR_ARG, "matvec: T=%d n=%d", T, n);
    MatvecArgs a{};
    a.nseg = n;
    a.x = x;
    a.in = in;
    const int n8 = in / 8;
    const int R = T == 1 ? mv_rows<1>() : mv_rows<2>();
    auto blocks_for = [&](int ks) {
        long long tot = 0;
        const int per_block = (MV_WARPS / ks) * R;
        for (int i = 0; i < n; i++) tot += (p[i].rows + per_block - 1) / per_block;
        return tot;
    };
    // split `in` over up to 4 warps while the grid is short of about 8 blocks per SM (a
    // measured optimum for streaming) and every slice still gives each lane at least two
    // 16-byte pieces
    int ks = 1;
    while (ks < 4 && blocks_for(ks) < 8LL * ctx->sm_count && n8 / (2 * ks) >= 64) ks *= 2;
    a.ks = ks;
    const int per_block = (MV_WARPS / ks) * R;
    long long tot = 0;
    for (int i = 0; i < n; i++) {
        a.seg[i] = MatvecSeg{p[i].W, p[i].y, p[i].rows, (p[i].rows + per_block - 1) / per_block};
        tot += a.seg[i].blocks;
    }
    if (tot == 0) return K3CUDA_OK;
    if (tot > 0x7fffffffLL) return set_error(K3CUDA_ERR_ARG, "matvec: grid too large");
    switch (T) {
        case 1: return launch_matvec<1>(ctx, a, wdt, (int)tot);
        case 2: return launch_matvec<2>(ctx, a, wdt, (int)tot);
        case 3: return launch_matvec<3>(ctx, a, wdt, (int)tot);
        case 4: return launch_matvec<4>(ctx, a, wdt, (int)tot);
        case 5: return launch_matvec<5>(ctx, a, wdt, (int)tot);
        case 6: return launch_matvec<6>(ctx, a, wdt, (int)tot);
        case 7: return launch_matvec<7>(ctx, a, wdt, (int)tot);
        default: return launch_matvec<8>(ctx, a, wdt, (int)tot);
    }
}

// hi = bf16(x), lo = bf16(x - hi): x = hi + lo to within 2^-16 |x|.
__global__ void split_bf16(__nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo,
                           const float *__restrict__ x, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

int split(k3cuda_ctx *ctx, __nv_bfloat16 *xs, const float *x, long long n) {
    const long long want = (n + 255) / 256;
    const int blocks = (int)(want < 8LL * ctx->sm_count ? want : 8LL * ctx->sm_count);
    split_bf16<<<blocks, 256, 0, ctx->stream>>>(xs, xs + n, x, n);
    return after_launch(ctx, "split_bf16");
}

// ------------------------------------------------------------ vector lane access
// A lane holds CPL consecutive channels of a head (D = 32 CPL, or D = 16 with lanes 16-31
// idle), moved with one CPL-wide load or store.
template <int CPL> struct fvec;
template <> struct fvec<1> {
    static __device__ __forceinline__ void ld(float v[1], const float *p) { v[0] = __ldg(p); }
    static __device__ __forceinline__ void st(float *p, const float v[1]) { *p = v[0]; }
};
template <> struct fvec<2> {
    static __device__ __forceinline__ void ld(float v[2], const float *p) {
        const float2 t = __ldg(reinterpret_cast<const float2 *>(p));
        v[0] = t.x; v[1] = t.y;
    }
    static __device__ __forceinline__ void st(float *p, const float v[2]) {
        *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
    }
};
template <> struct fvec<4> {
    static __device__ __forceinline__ void ld(float v[4], const float *p) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    }
    static __device__ __forceinline__ void st(float *p, const float v[4]) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
// the same for the recurrence's io type (fp32, or bf16 packed in pairs)
template <typename IO, int CPL> struct iovec {
    static __device__ __forceinline__ void ld(float v[CPL], const IO *p) { fvec<CPL>::ld(v, p); }
    static __device__ __forceinline__ void st(IO *p, const float v[CPL]) { fvec<CPL>::st(p, v); }
};
template <int CPL> struct iovec<__nv_bfloat16, CPL> {
    static __device__ __forceinline__ void ld(float v[CPL], const __nv_bfloat16 *p) {
        if constexpr (CPL == 1) {
            v[0] = __bfloat162float(*p);
        } else {
            unsigned int u[CPL / 2];
            if constexpr (CPL == 2) u[0] = *reinterpret_cast<const unsigned int *>(p);
            else { const uint2 t = *reinterpret_cast<const uint2 *>(p); u[0] = t.x; u[1] = t.y; }
#pragma unroll
            for (int m = 0; m < CPL / 2; m++) {
                v[2 * m] = __uint_as_float(u[m] << 16);
                v[2 * m + 1] = __uint_as_float(u[m] & 0xffff0000u);
            }
        }
    }
    static __device__ __forceinline__ void st(__nv_bfloat16 *p, const float v[CPL]) {
        if constexpr (CPL == 1) {
            *p = __float2bfloat16_rn(v[0]);
        } else {
            unsigned int u[CPL / 2];
#pragma unroll
            for (int m = 0; m < CPL / 2; m++) {
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * m], v[2 * m + 1]);
                u[m] = *reinterpret_cast<const unsigned int *>(&b2);
            }
            if constexpr (CPL == 2) *reinterpret_cast<unsigned int *>(p) = u[0];
            else *reinterpret_cast<uint2 *>(p) = make_uint2(u[0], u[1]);
        }
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------------ kda_layer_pre
// Grid (token tiles of LT, H, 4). z = 0, 1, 2: ShortConv + SiLU of the raw q, k, v
// projections of head h (k3_shortconv, k3_ops.c:133-165: taps oldest..newest, w[K-1] on the
// current input), then for q and k the L2 norm over the head's D channels (l2norm_,
// :845-851). z = 3: the decay chain g = lb * sigmoid(exp(A_log[h]) (z + dt_bias))
// (k3_kda_decay, :167-183, kept as log-decay) and beta = sigmoid(b x) (:902-903).
// Each warp owns TPW consecutive tokens and slides a window of K-1 + TPW raw rows through
// registers: K-1 history rows (older ones from the carried conv history) and its TPW rows,
// every load issued before the arithmetic. Lanes hold CPL channels each. The warp that owns
// token 0 is the only reader of the old conv history; it also writes the new one (the raw
// inputs of tokens T-K+1 .. T-1), after its reads.
constexpr int TPW = 8, LAYER_WARPS = 8, LT = TPW * LAYER_WARPS, LAYER_THREADS = 32 * LAYER_WARPS;

template <typename IO>
struct PreArgs {
    const float *y[3];   // raw projections q, k, v [T][P]
    const float *cw[3];  // conv taps [P][K]
    float *hist;         // conv histories [3][P][K-1], or null
    const float *z;      // low-rank decay input [T][P]
    const float *yb;     // beta logits [T][H]
    const float *A_log, *dt_bias;
    IO *out[3];          // recurrence q, k, v [T][P]
    float *g;            // log decay [T][P]
    float *beta;         // [T][H]
    int T, H, D;
    float lb;
};

template <typename IO, int CPL, int K>
__global__ void __launch_bounds__(LAYER_THREADS) kda_layer_pre(const __grid_constant__ PreArgs<IO> a) {
    pdl_trigger();
    pdl_wait();  // the projections come from the previous kernels
    constexpr int HIST = K - 1;
    const int s = blockIdx.z, h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t_a = blockIdx.x * LT + warp * TPW;
    const int D = a.D, P = a.H * D, c0 = lane * CPL;
    if (t_a >= a.T) return;  // whole warps only: no block-level synchronisation below
    const int nt = min(TPW, a.T - t_a);
    const bool on = c0 < D;  // lanes past the head's channels stay for the L2 reduction
    const size_t col = (size_t)h * D + (on ? c0 : 0);
    if (s == 3) {
        if (lane < nt) {
            const size_t i = (size_t)(t_a + lane) * a.H + h;
            a.beta[i] = dsigm(a.yb[i]);
        }
        if (!on) return;
        float dt[CPL], zv[TPW][CPL];
        fvec<CPL>::ld(dt, a.dt_bias + col);
#pragma unroll
        for (int tt = 0; tt < TPW; tt++)
            if (tt < nt) fvec<CPL>::ld(zv[tt], a.z + (size_t)(t_a + tt) * P + col);
        const float ea = expf(a.A_log[h]);
#pragma unroll
        for (int tt = 0; tt < TPW; tt++) {
            if (tt < nt) {
                float gv[CPL];
#pragma unroll
                for (int m = 0; m < CPL; m++) gv[m] = a.lb * dsigm(ea * (zv[tt][m] + dt[m]));
                fvec<CPL>::st(a.g + (size_t)(t_a + tt) * P + col, gv);
            }
        }
        return;
    }
    const float *y = a.y[s] + col;
    float *hs = (HIST > 0 && a.hist) ? a.hist + ((size_t)s * P + col) * HIST : nullptr;  // [CPL][HIST]
    // rows[r] = raw input of token t_a - HIST + r
    float rows[HIST + TPW][CPL];
#pragma unroll
    for (int r = 0; r < HIST + TPW; r++) {
        const int tok = t_a - HIST + r;
        if (tok >= 0) {
            if (tok < t_a + nt) fvec<CPL>::ld(rows[r], y + (size_t)tok * P);
        } else {
#pragma unroll
            for (int m = 0; m < CPL; m++) rows[r][m] = hs ? hs[m * HIST + (tok + HIST)] : 0.f;
        }
    }
    float wt[K][CPL];
#pragma unroll
    for (int m = 0; m < CPL; m++)
#pragma unroll
        for (int j = 0; j < K; j++) wt[j][m] = __ldg(a.cw[s] + (col + m) * K + j);
    if (t_a == 0 && hs && on) {
        // the new history: tokens T-HIST .. T-1, older than token 0 from the old history.
        // Slot j is written after slot T+j > j is read, so the shift is in place.
#pragma unroll
        for (int j = 0; j < HIST; j++) {
            const int tok = a.T - HIST + j;
            float v[CPL];
            if (tok >= 0) {
                fvec<CPL>::ld(v, y + (size_t)tok * P);
            } else {
#pragma unroll
                for (int m = 0; m < CPL; m++) v[m] = hs[m * HIST + (tok + HIST)];
            }
#pragma unroll
            for (int m = 0; m < CPL; m++) hs[m * HIST + j] = v[m];
        }
    }
    IO *out = a.out[s] + col;
#pragma unroll
    for (int tt = 0; tt < TPW; tt++) {
        if (tt >= nt) continue;
        float v[CPL], ss = 0.f;
#pragma unroll
        for (int m = 0; m < CPL; m++) {
            float acc = wt[HIST][m] * rows[tt + HIST][m];
#pragma unroll
            for (int j = 0; j < HIST; j++) acc += wt[j][m] * rows[tt + j][m];
            v[m] = acc * dsigm(acc);
            ss += on ? v[m] * v[m] : 0.f;
        }
        if (s < 2) {
            const float inv = rsqrtf(warp_sum(ss) + 1e-6f);
#pragma unroll
            for (int m = 0; m < CPL; m++) v[m] *= inv;
        }
        if (on) iovec<IO, CPL>::st(out + (size_t)(t_a + tt) * P, v);
    }
}

// ----------------------------------------------------------------- kda_layer_post
// ot = RMSNorm_head(o) * o_norm * sigmoid(g x) (k3_rmsnorm per head, then the gate,
// k3_ops.c:941-947), written as fp32 (the matvec input) and/or as the bf16 hi/lo split (the
// GEMM input). Warps own TPW tokens of one head, lanes CPL channels; loads first.
template <typename IO>
struct PostArgs {
    const IO *o;       // recurrence output [T][P]
    const float *gb;   // gate logits [T][P]
    const float *w;    // o_norm [D]
    float *ot;         // [T][P], or null
    __nv_bfloat16 *hi, *lo;  // [T][P] each, or null
    int T, H, D;
    float eps;
};

template <typename IO, int CPL>
__global__ void __launch_bounds__(LAYER_THREADS) kda_layer_post(const __grid_constant__ PostArgs<IO> a) {
    pdl_trigger();  // o_proj's CTAs may be scheduled while this kernel runs
    pdl_wait();
    const int h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t_a = blockIdx.x * LT + warp * TPW;
    const int D = a.D, P = a.H * D, c0 = lane * CPL;
    if (t_a >= a.T) return;
    const bool on = c0 < D;  // idle lanes still take part in the reductions
    const int nt = min(TPW, a.T - t_a);
    const size_t col = (size_t)h * D + (on ? c0 : 0);
    float wn[CPL], ov[TPW][CPL], gv[TPW][CPL];
    fvec<CPL>::ld(wn, a.w + (on ? c0 : 0));
#pragma unroll
    for (int tt = 0; tt < TPW; tt++) {
        if (tt < nt) {
            const size_t row = (size_t)(t_a + tt) * P + col;
            iovec<IO, CPL>::ld(ov[tt], a.o + row);
            fvec<CPL>::ld(gv[tt], a.gb + row);
        }
    }
#pragma unroll
    for (int tt = 0; tt < TPW; tt++) {
        if (tt >= nt) continue;
        float ss = 0.f;
#pragma unroll
        for (int m = 0; m < CPL; m++) ss += on ? ov[tt][m] * ov[tt][m] : 0.f;
        const float inv = rsqrtf(warp_sum(ss) / (float)D + a.eps);
        if (!on) continue;
        float r[CPL];
#pragma unroll
        for (int m = 0; m < CPL; m++) {
            r[m] = wn[m] * ov[tt][m] * inv;
            r[m] *= dsigm(gv[tt][m]);
        }
        const size_t row = (size_t)(t_a + tt) * P + col;
        if (a.ot) fvec<CPL>::st(a.ot + row, r);
        if (a.hi) {
            float hv[CPL], lv[CPL];
#pragma unroll
            for (int m = 0; m < CPL; m++) {
                hv[m] = __bfloat162float(__float2bfloat16_rn(r[m]));
                lv[m] = r[m] - hv[m];
            }
            iovec<__nv_bfloat16, CPL>::st(a.hi + row, hv);
            iovec<__nv_bfloat16, CPL>::st(a.lo + row, lv);
        }
    }
}

// ----------------------------------------------------------------- workspace plan
static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

struct LayerPlan {
    // byte offsets into the workspace
    size_t yq, yk, yv, z, gb, yb, fa, rq, rk, rv, g, beta, o, xs, fas, s0, pre, total;
    size_t pre_bytes;
    bool gemm_path, split;
    int io_size;
};

static int plan_layer(int T, int E, int H, int D, int K, int wdt, int io_dtype, LayerPlan *p) {
    (void)K;
    const size_t P = (size_t)H * D, TP = (size_t)T * P;
    const int es = io_dtype == K3CUDA_BF16 ? 2 : 4;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += al256(bytes); return o; };
    p->gemm_path = T > MV_MAXT;
    p->split = p->gemm_path && wdt == K3CUDA_BF16;
    p->io_size = es;
    p->yq = take(TP * 4);  // later the post kernel's ot
    p->yk = take(TP * 4);  // later ot's bf16 hi/lo split (same bytes)
    p->yv = take(TP * 4);
    p->z = take(TP * 4);
    p->gb = take(TP * 4);
    p->yb = take((size_t)T * H * 4);
    p->fa = take((size_t)T * D * 4);
    p->rq = take(TP * es);
    p->rk = take(TP * es);
    p->rv = take(TP * es);
    p->g = take(TP * 4);
    p->beta = take((size_t)T * H * 4);
    p->o = take(TP * es);
    p->xs = p->split ? take((size_t)2 * T * E * 2) : 0;
    p->fas = p->split ? take((size_t)2 * T * D * 2) : 0;
    p->s0 = take(P * D * 4);
    p->pre_bytes = 0;
    if (T > 1 && (D == 64 || D == 128)) {
        const int cu[2] = {0, T};
        int rc = k3cuda_kda_prefill_workspace(cu, 1, H, D, D, 64, &p->pre_bytes);
        if (rc) return rc;
    }
    p->pre = take(p->pre_bytes);
    p->total = off;
    return K3CUDA_OK;
}

static int layer_shape_ok(int T, int E, int H, int D, int K, int wdt, int io_dtype) {
    K3_ARG_CHECK(T >= 0 && E >= 8 && H >= 1 && D >= 16 && K >= 1, "kda_layer: bad shape T=%d "
                 "E=%d H=%d D=%d K=%d", T, E, H, D, K);
    K3_ARG_CHECK(wdt == K3CUDA_F32 || wdt == K3CUDA_BF16, "kda_layer: bad wdt %d", wdt);
    K3_ARG_CHECK(io_dtype == K3CUDA_F32 || io_dtype == K3CUDA_BF16, "kda_layer: bad io_dtype %d",
                 io_dtype);
    if (E % 8 || D % 16 || D > 128 || K > 4)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "kda_layer: E=%d D=%d K=%d not built (E %% 8 "
                         "== 0, D %% 16 == 0, D <= 128, K <= 4)", E, D, K);
    return K3CUDA_OK;
}

template <typename IO, int CPL>
static int launch_pre_k(k3cuda_ctx *ctx, const PreArgs<IO> &a, int K, dim3 grid) {
    const dim3 blk(LAYER_THREADS);
    const char *nm = "kda_layer_pre";
    switch (K) {
        case 1: return launch_pdl(ctx, ctx->stream, nm, kda_layer_pre<IO, CPL, 1>, grid, blk, 0, a);
        case 2: return launch_pdl(ctx, ctx->stream, nm, kda_layer_pre<IO, CPL, 2>, grid, blk, 0, a);
        case 3: return launch_pdl(ctx, ctx->stream, nm, kda_layer_pre<IO, CPL, 3>, grid, blk, 0, a);
        default: return launch_pdl(ctx, ctx->stream, nm, kda_layer_pre<IO, CPL, 4>, grid, blk, 0, a);
    }
}

template <typename IO>
static int launch_pre(k3cuda_ctx *ctx, const PreArgs<IO> &a, int D, int K, dim3 grid) {
    if (D <= 32) return launch_pre_k<IO, 1>(ctx, a, K, grid);
    if (D <= 64) return launch_pre_k<IO, 2>(ctx, a, K, grid);
    return launch_pre_k<IO, 4>(ctx, a, K, grid);
}

// One projection: matvec (T <= 8) or GEMM; xs is x's bf16 split when the GEMM needs it.
int project(k3cuda_ctx *ctx, float *y, const float *x, const __nv_bfloat16 *xs,
                   const void *W, int wdt, int T, int in, int out) {
    if (T <= MV_MAXT) {
        const Proj p{W, y, out};
        return matvec(ctx, x, T, in, &p, 1, wdt);
    }
    return gemm(ctx, y, x, xs, W, wdt, T, in, out);
}

template <typename IO>
static int layer_core(k3cuda_ctx *ctx, float *out, const float *x, const k3cuda_kda_weights *w,
                      int T, int E, int H, int D, int K, float lb, float eps, float *state,
                      int io_dtype, char *ws, const LayerPlan &pl) {
    const int P = H * D, hist = K - 1, wdt = w->wdt;
    float *yq = (float *)(ws + pl.yq), *yk = (float *)(ws + pl.yk), *yv = (float *)(ws + pl.yv);
    float *z = (float *)(ws + pl.z), *gb = (float *)(ws + pl.gb), *yb = (float *)(ws + pl.yb);
    float *fa = (float *)(ws + pl.fa), *g = (float *)(ws + pl.g), *beta = (float *)(ws + pl.beta);
    IO *rq = (IO *)(ws + pl.rq), *rk = (IO *)(ws + pl.rk), *rv = (IO *)(ws + pl.rv);
    IO *o = (IO *)(ws + pl.o);
    __nv_bfloat16 *xs = pl.split ? (__nv_bfloat16 *)(ws + pl.xs) : nullptr;
    __nv_bfloat16 *fas = pl.split ? (__nv_bfloat16 *)(ws + pl.fas) : nullptr;
    int rc;
    // 1. projections (and the gate's g x, which reads the same x)
    bool forked = false;
    if (!pl.gemm_path) {
        const Proj first[5] = {{w->q, yq, P}, {w->k, yk, P}, {w->v, yv, P},
                               {w->b, yb, H}, {w->f_a, fa, D}};
        // The gate projection (needed at step 8) streams on the side stream from the start:
        // its blocks fill the tail of the main projection launch and it finishes while the
        // chain of small kernels of steps 2-6 runs on the main stream (forking it after the
        // main projection instead left step 7 waiting for it: 0.172 vs 0.161 ms per token).
        K3_CUDA_TRY(cudaEventRecord(ctx->ev_fork, ctx->stream));
        K3_CUDA_TRY(cudaStreamWaitEvent(ctx->aux, ctx->ev_fork, 0));
        cudaStream_t main_stream = ctx->stream;
        ctx->stream = ctx->aux;
        const Proj gate{w->g, gb, P};
        rc = matvec(ctx, x, T, E, &gate, 1, wdt);
        ctx->stream = main_stream;
        if (rc) return rc;
        K3_CUDA_TRY(cudaEventRecord(ctx->ev_join, ctx->aux));
        forked = true;
        if ((rc = matvec(ctx, x, T, E, first, 5, wdt))) return rc;
    } else {
        if (pl.split && (rc = split(ctx, xs, x, (long long)T * E))) return rc;
        const Proj first[6] = {{w->q, yq, P}, {w->k, yk, P}, {w->v, yv, P},
                               {w->g, gb, P}, {w->b, yb, H}, {w->f_a, fa, D}};
        for (const Proj &p : first)
            if ((rc = gemm(ctx, p.y, x, xs, p.W, wdt, T, E, p.rows))) return rc;
        if (pl.split && (rc = split(ctx, fas, fa, (long long)T * D))) return rc;
    }
    if ((rc = project(ctx, z, fa, fas, w->f_b, wdt, T, D, P))) return rc;
    // 2-5. conv + SiLU, L2, decay, beta
    {
        PreArgs<IO> a{};
        a.y[0] = yq; a.y[1] = yk; a.y[2] = yv;
        a.cw[0] = w->q_conv; a.cw[1] = w->k_conv; a.cw[2] = w->v_conv;
        a.hist = state && hist > 0 ? state + (size_t)H * D * D : nullptr;
        a.z = z; a.yb = yb; a.A_log = w->A_log; a.dt_bias = w->dt_bias;
        a.out[0] = rq; a.out[1] = rk; a.out[2] = rv;
        a.g = g; a.beta = beta;
        a.T = T; a.H = H; a.D = D; a.lb = lb;
        dim3 grid((unsigned)((T + LT - 1) / LT), (unsigned)H, 4);
        if ((rc = launch_pre(ctx, a, D, K, grid))) return rc;
    }
    // 6. recurrence
    float *S = state;
    if (!S) {
        S = (float *)(ws + pl.s0);
        K3_CUDA_TRY(cudaMemsetAsync(S, 0, (size_t)P * D * sizeof(float), ctx->stream));
    }
    const float qs = 1.0f / sqrtf((float)D);
    if (T == 1 || pl.pre_bytes == 0) {
        for (int t = 0; t < T; t++) {
            const size_t off = (size_t)t * P;
            rc = k3cuda_kda_decode(ctx, S, o + off, rq + off, rk + off, rv + off, g + off,
                                   beta + (size_t)t * H, 1, H, D, D, qs, io_dtype,
                                   K3CUDA_GATE_LOG);
            if (rc) return rc;
        }
    } else {
        const int cu[2] = {0, T};
        rc = k3cuda_kda_prefill(ctx, S, o, rq, rk, rv, g, beta, cu, 1, H, D, D, qs, io_dtype,
                                K3CUDA_GATE_LOG, 64, ws + pl.pre, pl.pre_bytes);
        if (rc) return rc;
    }
    // 7/8. head RMSNorm, then the gate (ot reuses yq, its split reuses yk)
    if (forked) K3_CUDA_TRY(cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
    float *ot = yq;
    __nv_bfloat16 *ots = pl.split ? (__nv_bfloat16 *)yk : nullptr;
    {
        PostArgs<IO> a{};
        a.o = o; a.gb = gb; a.w = w->o_norm; a.ot = pl.split ? nullptr : ot;
        a.hi = ots; a.lo = ots ? ots + (size_t)T * P : nullptr;
        a.T = T; a.H = H; a.D = D; a.eps = eps;
        dim3 grid((unsigned)((T + LT - 1) / LT), (unsigned)H);
        if (D <= 32) kda_layer_post<IO, 1><<<grid, LAYER_THREADS, 0, ctx->stream>>>(a);
        else if (D <= 64) kda_layer_post<IO, 2><<<grid, LAYER_THREADS, 0, ctx->stream>>>(a);
        else kda_layer_post<IO, 4><<<grid, LAYER_THREADS, 0, ctx->stream>>>(a);
        if ((rc = after_launch(ctx, "kda_layer_post"))) return rc;
    }
    // 9. o_proj
    return project(ctx, out, ot, ots, w->o, wdt, T, P, E);
}

}  // namespace k3

using namespace k3;



extern "C" int k3cuda_matmul_workspace(int T, int in, int wdt, size_t *bytes) {
    K3_ARG_CHECK(bytes && T >= 0 && in >= 0, "bad matmul workspace query");
    K3_ARG_CHECK(wdt == K3CUDA_F32 || wdt == K3CUDA_BF16, "matmul: bad wdt %d", wdt);
    *bytes = (T > MV_MAXT && wdt == K3CUDA_BF16) ? al256((size_t)2 * T * in * 2) : 0;
    return K3CUDA_OK;
}

extern "C" int k3cuda_matmul(k3cuda_ctx *ctx, float *y, const float *x, const void *W, int wdt,
                             int in, int out, int T, void *workspace, size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    size_t need = 0;
    if ((rc = k3cuda_matmul_workspace(T, in, wdt, &need))) return rc;
    K3_ARG_CHECK(out >= 0, "matmul: out=%d", out);
    if (T == 0 || out == 0) return K3CUDA_OK;
    K3_ARG_CHECK(y && x && W, "matmul: null pointer");
    if (in % 8) return set_error(K3CUDA_ERR_UNSUPPORTED, "matmul: in=%d not a multiple of 8", in);
    K3_ARG_CHECK(aligned(y, 16) && aligned(x, 16) && aligned(W, 16),
                 "matmul: x, W, y must be 16-byte aligned");
    if (workspace_bytes < need || (need && !workspace))
        return set_error(K3CUDA_ERR_WORKSPACE, "matmul: workspace %zu < %zu bytes",
                         workspace_bytes, need);
    __nv_bfloat16 *xs = need ? (__nv_bfloat16 *)workspace : nullptr;
    if (xs && (rc = split(ctx, xs, x, (long long)T * in))) return rc;
    return project(ctx, y, x, xs, W, wdt, T, in, out);
}

extern "C" int k3cuda_kda_layer_workspace(int T, int E, int H, int D, int K, int wdt,
                                          int io_dtype, size_t *bytes) {
    K3_ARG_CHECK(bytes, "null bytes");
    int rc = layer_shape_ok(T, E, H, D, K, wdt, io_dtype);
    if (rc) return rc;
    LayerPlan p;
    if ((rc = plan_layer(T, E, H, D, K, wdt, io_dtype, &p))) return rc;
    *bytes = p.total;
    return K3CUDA_OK;
}

extern "C" int k3cuda_kda_layer(k3cuda_ctx *ctx, float *out, const float *x,
                                const k3cuda_kda_weights *w, int T, int E, int H, int D, int K,
                                float gate_lb, float rms_eps, float *state, int io_dtype,
                                void *workspace, size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(w, "kda_layer: null weights");
    if ((rc = layer_shape_ok(T, E, H, D, K, w->wdt, io_dtype))) return rc;
    if (T == 0) return K3CUDA_OK;
    K3_ARG_CHECK(out && x && w->q && w->k && w->v && w->q_conv && w->k_conv && w->v_conv &&
                 w->f_a && w->f_b && w->A_log && w->dt_bias && w->b && w->g && w->o_norm &&
                 w->o, "kda_layer: null pointer");
    const void *vec[] = {out, x, w->q, w->k, w->v, w->f_a, w->f_b, w->b, w->g, w->o,
                         w->dt_bias, w->o_norm};
    for (const void *p : vec)
        K3_ARG_CHECK(aligned(p, 16), "kda_layer: x, out, the projection weights, dt_bias and "
                     "o_norm must be 16-byte aligned");
    K3_ARG_CHECK(aligned(state, 16), "kda_layer: state must be 16-byte aligned");
    LayerPlan pl;
    if ((rc = plan_layer(T, E, H, D, K, w->wdt, io_dtype, &pl))) return rc;
    if (workspace_bytes < pl.total || !workspace)
        return set_error(K3CUDA_ERR_WORKSPACE, "kda_layer: workspace %zu < %zu bytes",
                         workspace_bytes, pl.total);
    K3_ARG_CHECK(aligned(workspace, 256), "kda_layer: workspace must be 256-byte aligned");
    if (io_dtype == K3CUDA_BF16)
        return layer_core<__nv_bfloat16>(ctx, out, x, w, T, E, H, D, K, gate_lb, rms_eps, state,
                                         io_dtype, (char *)workspace, pl);
    return layer_core<float>(ctx, out, x, w, T, E, H, D, K, gate_lb, rms_eps, state, io_dtype,
                             (char *)workspace, pl);
}
