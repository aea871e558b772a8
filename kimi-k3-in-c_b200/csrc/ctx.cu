// ctx.cu -- context, memory, events and error reporting of libk3cuda.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <initializer_list>
#include <mutex>

#include "internal.cuh"
#include "sm100.cuh"

namespace k3 {

// One CTA waits on a barrier that nothing arrives on, under the context's wait bound: the
// timeout path of every pipelined kernel (error word set, the kernel returns) without a
// fault, a trap or an unbounded spin.
__global__ void wait_selftest(unsigned *err) {
    using namespace sm100;
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, err, 0x5E1Fu);
}

static thread_local char g_err[1024] = "";

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_err[0] = 0; }

int enter(k3cuda_ctx *ctx) {
    if (!ctx) return set_error(K3CUDA_ERR_ARG, "null context");
    K3_CUDA_TRY(cudaSetDevice(ctx->device));
    return K3CUDA_OK;
}

int after_launch(k3cuda_ctx *ctx, const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(K3CUDA_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    ctx->launches++;
    return K3CUDA_OK;
}

int set_smem(const void *func, int bytes) {
    struct Ent { const void *f; int dev, bytes; };
    static Ent tab[128];
    static int n = 0;
    static std::mutex mu;
    int dev = 0;
    K3_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < n; i++)
        if (tab[i].f == func && tab[i].dev == dev && tab[i].bytes >= bytes) return K3CUDA_OK;
    K3_CUDA_TRY(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    if (n < 128) tab[n++] = Ent{func, dev, bytes};
    return K3CUDA_OK;
}

constexpr int PIN_SLOTS = 16;
constexpr size_t PIN_SLOT = 512u << 10;

int stage_h2d(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (bytes == 0) return K3CUDA_OK;
    if (bytes > PIN_SLOT) {
        K3_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
        return K3CUDA_OK;
    }
    if (!ctx->pin) {
        K3_CUDA_TRY(cudaMallocHost((void **)&ctx->pin, PIN_SLOTS * PIN_SLOT));
        for (int i = 0; i < PIN_SLOTS; i++) {
            K3_CUDA_TRY(cudaEventCreateWithFlags(&ctx->pin_ev[i], cudaEventDisableTiming));
            ctx->pin_used[i] = false;
        }
    }
    const int slot = ctx->pin_next;
    ctx->pin_next = (slot + 1) % PIN_SLOTS;
    if (ctx->pin_used[slot]) K3_CUDA_TRY(cudaEventSynchronize(ctx->pin_ev[slot]));
    unsigned char *buf = ctx->pin + (size_t)slot * PIN_SLOT;
    memcpy(buf, src, bytes);
    K3_CUDA_TRY(cudaMemcpyAsync(dst, buf, bytes, cudaMemcpyHostToDevice, ctx->stream));
    K3_CUDA_TRY(cudaEventRecord(ctx->pin_ev[slot], ctx->stream));
    ctx->pin_used[slot] = true;
    return K3CUDA_OK;
}

}  // namespace k3

using namespace k3;

extern "C" {

const char *k3cuda_last_error(void) { return g_err; }

int k3cuda_device_count(int *count) {
    K3_ARG_CHECK(count, "null count");
    K3_CUDA_TRY(cudaGetDeviceCount(count));
    return K3CUDA_OK;
}

int k3cuda_init(int device, k3cuda_ctx **out) {
    K3_ARG_CHECK(out, "null output pointer");
    *out = nullptr;
    int n = 0;
    K3_CUDA_TRY(cudaGetDeviceCount(&n));
    K3_ARG_CHECK(device >= 0 && device < n, "device %d out of range (%d devices)", device, n);
    K3_CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop;
    K3_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return set_error(K3CUDA_ERR_UNSUPPORTED,
                         "device %d is sm_%d%d; libk3cuda is built for sm_100a (B200) only",
                         device, prop.major, prop.minor);
    k3cuda_ctx *c = (k3cuda_ctx *)calloc(1, sizeof(k3cuda_ctx));
    if (!c) return set_error(K3CUDA_ERR_ARG, "out of host memory");
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    for (int i = 0; e == cudaSuccess && i < K3CUDA_MAX_EVENTS; i++)
        e = cudaEventCreate(&c->events[i]);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->aux, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->cp_in, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->cp_out, cudaStreamNonBlocking);
    cudaEvent_t *evs[] = {&c->ev_cp_start, &c->ev_cp_in_done, &c->ev_cp_out_done};
    for (cudaEvent_t *ev : evs)
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
    for (int i = 0; e == cudaSuccess && i < K3CUDA_HOST_SLICES; i++) {
        e = cudaEventCreateWithFlags(&c->ev_in[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_k[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaMalloc((void **)&c->err_word, 256);
    if (e == cudaSuccess) e = cudaMemset(c->err_word, 0, 256);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_fence, cudaEventDisableTiming);
    c->comm_timeout_ms = 60000;
    if (e != cudaSuccess) {
        k3cuda_shutdown(c);  // releases whatever was created (every member starts out null)
        return set_error(K3CUDA_ERR_CUDA, "context creation failed: %s", cudaGetErrorString(e));
    }
    *out = c;
    clear_error();
    return K3CUDA_OK;
}

int k3cuda_comm_destroy_internal(k3cuda_ctx *ctx);  // comm.cu

int k3cuda_shutdown(k3cuda_ctx *ctx) {
    if (!ctx) return K3CUDA_OK;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    k3cuda_comm_destroy_internal(ctx);
    for (int i = 0; i < K3CUDA_MAX_EVENTS; i++)
        if (ctx->events[i]) cudaEventDestroy(ctx->events[i]);
    if (ctx->flush_buf) cudaFree(ctx->flush_buf);
    if (ctx->err_word) cudaFree(ctx->err_word);
    if (ctx->pin) {
        for (int i = 0; i < PIN_SLOTS; i++)
            if (ctx->pin_ev[i]) cudaEventDestroy(ctx->pin_ev[i]);
        cudaFreeHost(ctx->pin);
    }
    if (ctx->ev_fence) cudaEventDestroy(ctx->ev_fence);
    if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
    if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
    if (ctx->aux) cudaStreamDestroy(ctx->aux);
    for (cudaStream_t cs : {ctx->cp_in, ctx->cp_out})
        if (cs) {
            cudaStreamSynchronize(cs);
            cudaStreamDestroy(cs);
        }
    for (cudaEvent_t ev : {ctx->ev_cp_start, ctx->ev_cp_in_done, ctx->ev_cp_out_done})
        if (ev) cudaEventDestroy(ev);
    for (int i = 0; i < K3CUDA_HOST_SLICES; i++) {
        if (ctx->ev_in[i]) cudaEventDestroy(ctx->ev_in[i]);
        if (ctx->ev_k[i]) cudaEventDestroy(ctx->ev_k[i]);
    }
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    free(ctx);
    return K3CUDA_OK;
}

int k3cuda_sync(k3cuda_ctx *ctx) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (ctx->nccl_comm) {
        // the stream may hold collectives: wait under the communicator's deadline
        rc = comm_wait_stream(ctx);
        if (rc) return rc;
    }
    K3_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    // a kernel whose bounded wait gave up leaves its code in the error word
    unsigned code = 0;
    K3_CUDA_TRY(cudaMemcpy(&code, ctx->err_word, sizeof code, cudaMemcpyDeviceToHost));
    if (code) {
        K3_CUDA_TRY(cudaMemset(ctx->err_word, 0, sizeof code));
        return set_error(K3CUDA_ERR_TIMEOUT, "a device-side wait timed out (code 0x%x)", code);
    }
    return K3CUDA_OK;
}

void *k3cuda_stream(k3cuda_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int k3cuda_set_wait_limit(k3cuda_ctx *ctx, long long cycles) {
    int rc = enter(ctx);
    if (rc) return rc;
    // byte 8 of the error block, read by every bounded wait (stream-ordered, so kernels
    // already queued keep the bound they were launched under)
    const long long v = cycles > 0 ? cycles : 0;
    K3_CUDA_TRY(cudaMemcpyAsync((char *)ctx->err_word + 8, &v, sizeof v, cudaMemcpyHostToDevice,
                                ctx->stream));
    K3_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    return K3CUDA_OK;
}

int k3cuda_wait_selftest(k3cuda_ctx *ctx) {
    int rc = enter(ctx);
    if (rc) return rc;
    wait_selftest<<<1, 32, 0, ctx->stream>>>(ctx->err_word);
    return after_launch(ctx, "wait_selftest");
}

int k3cuda_malloc(k3cuda_ctx *ctx, void **dptr, size_t bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(dptr, "null output pointer");
    *dptr = nullptr;
    if (bytes == 0) return K3CUDA_OK;
    K3_CUDA_TRY(cudaMalloc(dptr, bytes));
    return K3CUDA_OK;
}

int k3cuda_free(k3cuda_ctx *ctx, void *dptr) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (dptr) K3_CUDA_TRY(cudaFree(dptr));
    return K3CUDA_OK;
}

int k3cuda_host_alloc(k3cuda_ctx *ctx, void **hptr, size_t bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(hptr, "null output pointer");
    *hptr = nullptr;
    if (bytes == 0) return K3CUDA_OK;
    K3_CUDA_TRY(cudaMallocHost(hptr, bytes));
    return K3CUDA_OK;
}

int k3cuda_host_free(k3cuda_ctx *ctx, void *hptr) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (hptr) K3_CUDA_TRY(cudaFreeHost(hptr));
    return K3CUDA_OK;
}

static int copy(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes, cudaMemcpyKind kind) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (bytes == 0) return K3CUDA_OK;
    K3_ARG_CHECK(dst && src, "null copy pointer");
    K3_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, kind, ctx->stream));
    return K3CUDA_OK;
}

int k3cuda_memcpy_h2d(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes) {
    return copy(ctx, dst, src, bytes, cudaMemcpyHostToDevice);
}
int k3cuda_memcpy_d2h(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes) {
    return copy(ctx, dst, src, bytes, cudaMemcpyDeviceToHost);
}
int k3cuda_memcpy_d2d(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes) {
    return copy(ctx, dst, src, bytes, cudaMemcpyDeviceToDevice);
}

int k3cuda_memset(k3cuda_ctx *ctx, void *dptr, int value, size_t bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (bytes == 0) return K3CUDA_OK;
    K3_ARG_CHECK(dptr, "null pointer");
    K3_CUDA_TRY(cudaMemsetAsync(dptr, value, bytes, ctx->stream));
    return K3CUDA_OK;
}

int k3cuda_event_record(k3cuda_ctx *ctx, int slot) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(slot >= 0 && slot < K3CUDA_MAX_EVENTS, "event slot %d out of range", slot);
    K3_CUDA_TRY(cudaEventRecord(ctx->events[slot], ctx->stream));
    return K3CUDA_OK;
}

int k3cuda_event_elapsed(k3cuda_ctx *ctx, int a, int b, float *ms) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(a >= 0 && a < K3CUDA_MAX_EVENTS && b >= 0 && b < K3CUDA_MAX_EVENTS && ms,
                 "bad event slots");
    K3_CUDA_TRY(cudaEventSynchronize(ctx->events[b]));
    K3_CUDA_TRY(cudaEventElapsedTime(ms, ctx->events[a], ctx->events[b]));
    return K3CUDA_OK;
}

long long k3cuda_launch_count(k3cuda_ctx *ctx) { return ctx ? ctx->launches : 0; }

int k3cuda_flush_l2(k3cuda_ctx *ctx) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!ctx->flush_buf) {
        int l2 = 0;
        K3_CUDA_TRY(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, ctx->device));
        ctx->flush_bytes = (size_t)l2 * 2 + (64u << 20);
        K3_CUDA_TRY(cudaMalloc(&ctx->flush_buf, ctx->flush_bytes));
    }
    K3_CUDA_TRY(cudaMemsetAsync(ctx->flush_buf, 0, ctx->flush_bytes, ctx->stream));
    return K3CUDA_OK;
}

}  // extern "C"
