// internal.cuh -- shared state and helpers of libk3cuda (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include "k3cuda.h"

struct k3cuda_ctx {
    int device;
    int sm_count;
    cudaStream_t stream;
    cudaEvent_t events[K3CUDA_MAX_EVENTS];
    long long launches;
    void *flush_buf;
    size_t flush_bytes;
    unsigned int *err_word;     // device word set by bounded waits that gave up
    // NCCL (opaque; see comm.cu)
    void *nccl_comm;
    int nranks, rank;
    int comm_timeout_ms;        // host deadline of every wait that involves the communicator
    int comm_failed;            // the communicator was aborted (a peer left or timed out)
    cudaEvent_t ev_fence;       // completion of the last cross-rank fence
    // every rank's registered [T][H][dv] output, mapped into this process (comm.cu)
    void *full_out[K3CUDA_MAX_RANKS];
    void *full_base[K3CUDA_MAX_RANKS];   // peer allocations opened by IPC (to close)
    size_t full_bytes;
    int *sync_word;             // device int for the cross-rank ordering all-reduce
    void *peer_table;           // device copy of the peers' full-buffer addresses
    cudaStream_t aux;           // side stream for work that overlaps the main stream's
    cudaEvent_t ev_fork, ev_join;  // (forked from and joined back into `stream`)
    // page-locked ring for the small per-call host tables (stage_h2d)
    unsigned char *pin;
    int pin_next;
    cudaEvent_t pin_ev[16];
    bool pin_used[16];
    // host-buffer entry points: inputs come in on cp_in, results go out on cp_out, slice by
    // slice, both forked from and joined back into `stream`
    cudaStream_t cp_in, cp_out;
    cudaEvent_t ev_cp_start, ev_cp_in_done, ev_cp_out_done;
    cudaEvent_t ev_in[K3CUDA_HOST_SLICES], ev_k[K3CUDA_HOST_SLICES];
};

namespace k3 {
// Output of a head-sharded prefill written straight into every rank's full
// [T][H_total][dv] bf16 buffer (rank-local heads at head0..head0+H_local-1).
struct GatherOut {
    __nv_bfloat16 *ptr[K3CUDA_MAX_RANKS];
    int n;        // ranks (0: write the local output instead)
    int head0;    // first head of this rank in the full layout
    int H_total;
};
}  // namespace k3

namespace k3 {

// Projections. split (kda_layer.cu): hi = bf16(x), lo = bf16(x - hi) into xs [2][n].
// gemm (gemm.cu): y [T][out] = x [T][in] W^T; W bf16 on tcgen05 over xs (the bf16 split of
// x), or fp32 (and untiled shapes) on the CUDA cores.
int split(k3cuda_ctx *ctx, __nv_bfloat16 *xs, const float *x, long long n);
int gemm(k3cuda_ctx *ctx, float *y, const float *x, const __nv_bfloat16 *xs, const void *W,
         int wdt, int T, int in, int out);
// One weight matrix [rows][in] of a projection table and its output [T][rows].
struct Proj {
    const void *W;
    float *y;
    int rows;
};
constexpr int PROJ_MAXT = 8;  // up to this many activation rows the projections stream W
// n (<= 8) projections of the same x [T][in], T <= PROJ_MAXT, in one launch
int matvec(k3cuda_ctx *ctx, const float *x, int T, int in, const Proj *p, int n, int wdt);
// one projection: streaming (T <= PROJ_MAXT) or GEMM (xs: x's bf16 split for bf16 W)
int project(k3cuda_ctx *ctx, float *y, const float *x, const __nv_bfloat16 *xs, const void *W,
            int wdt, int T, int in, int out);
// MLA attention of T queries at positions cached.. of one sequence, W_UK/W_UV in kv_b
// (mla_decode.cu)
int mla_attend_kvb(k3cuda_ctx *ctx, float *acc, const void *q_nope, const void *q_rope,
                   const void *latent, const void *rope, const void *kv_b, int T, int cached,
                   int cap, int H, float scale, void *workspace, size_t workspace_bytes);
size_t mla_attend_kvb_workspace(int T, int cached, int H);

// Host -> device copy of a small per-call table on the context's stream without the
// stream synchronisation a pageable source may cost: the bytes go through a slot of a
// page-locked ring (16 slots of 512 KB; a slot is reused once the copy that last read it
// has completed). Larger tables fall back to a plain copy.
int stage_h2d(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes);

// cudaFuncSetAttribute(func, MaxDynamicSharedMemorySize, bytes) on the current device,
// skipped when this (function, device) pair already has at least `bytes`.
int set_smem(const void *func, int bytes);
template <typename F> inline int set_smem(F *func, int bytes) {
    return set_smem(reinterpret_cast<const void *>(func), bytes);
}

// Multi-rank state (comm.cu). comm_wait_stream: wait for the context's stream under the
// communicator's deadline, polling NCCL's asynchronous error; a deadline that passes or an
// error aborts the communicator (K3CUDA_ERR_TIMEOUT / K3CUDA_ERR_NCCL). Returns K3CUDA_OK
// at once when the context has no communicator.
int comm_wait_stream(k3cuda_ctx *ctx);

// Record an error message for the calling thread; returns `code`.
int set_error(int code, const char *fmt, ...);
void clear_error();

// Make ctx->device current; returns K3CUDA_OK or an error.
int enter(k3cuda_ctx *ctx);

// Check the last launch, count it, and convert failures.
int after_launch(k3cuda_ctx *ctx, const char *what);

#define K3_CUDA_TRY(expr)                                                                  \
    do {                                                                                   \
        cudaError_t _e = (expr);                                                           \
        if (_e != cudaSuccess)                                                             \
            return ::k3::set_error(K3CUDA_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,        \
                                   cudaGetErrorString(_e), __FILE__, __LINE__);            \
    } while (0)

#define K3_ARG_CHECK(cond, ...)                                                            \
    do {                                                                                   \
        if (!(cond)) return ::k3::set_error(K3CUDA_ERR_ARG, __VA_ARGS__);                  \
    } while (0)

inline bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

// ------------------------------------------------ programmatic dependent launch (PDL)
// The kernels of a dependent chain (a layer's T <= 8 path) are launched with programmatic
// stream serialization: the next kernel's CTAs are scheduled while the current one
// finishes, run their independent prologue (weight loads), and wait in pdl_wait() until the
// previous kernel has completed and its writes are visible. A kernel calls pdl_wait() before
// it reads anything an earlier kernel wrote and before its first global write; launched
// without the attribute, pdl_wait() returns at once. pdl_trigger() lets the next kernel be
// scheduled once every CTA of this one has issued it (its pdl_wait still waits for the end).
// A kernel that does not call pdl_trigger lets its successor start only when it has finished,
// as a plain launch would. The projections read weights before their pdl_wait, which is safe
// because no kernel that calls pdl_trigger writes a weight matrix; a kernel that produces
// weights (the MXFP4 expansion, the kv_b conversion) must keep not calling it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
int launch_pdl(k3cuda_ctx *ctx, cudaStream_t st, const char *what, void (*kern)(KArgs...),
               dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    if (e != cudaSuccess)
        return set_error(K3CUDA_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return after_launch(ctx, what);
}

// ------------------------------------------------------------------ element access
template <typename T> struct io;
template <> struct io<float> {
    static __device__ __forceinline__ float ld(const float *p) { return *p; }
    static __device__ __forceinline__ void st(float *p, float x) { *p = x; }
};
template <> struct io<__nv_bfloat16> {
    static __device__ __forceinline__ float ld(const __nv_bfloat16 *p) {
        return __bfloat162float(*p);
    }
    static __device__ __forceinline__ void st(__nv_bfloat16 *p, float x) {
        *p = __float2bfloat16_rn(x);
    }
};

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

}  // namespace k3
