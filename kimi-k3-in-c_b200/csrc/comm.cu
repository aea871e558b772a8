// comm.cu -- head-sharded output exchange over NVLink (NCCL all-gather + head interleave).
//
// The reference engine is single-process and has no communicator; this is the one
// exchange head sharding adds. Each rank holds its H_local heads of the KDA output as
// [T][H_local][dv]; ncclAllGather places the R slabs rank-major in the workspace, and
// head_interleave writes them to [T][R*H_local][dv] so rank r's heads land at
// r*H_local.. (the layout o_proj consumes, k3_ops.c:941-949).
//
// NCCL is opened with dlopen at first use (libnccl.so.2, whichever copy the process
// already has or the system one), so the library loads and runs single-GPU without it.
//
// Failure handling. The communicator is non-blocking: no NCCL call waits on the host.
// Every host wait that involves it (initialisation, a fence the host must see complete,
// k3cuda_sync of a context with a communicator) polls ncclCommGetAsyncError under a
// deadline (k3cuda_comm_set_timeout, 60 s by default). An asynchronous error, or a peer that
// never reaches a collective, ends in ncclCommAbort and a K3CUDA_ERR_NCCL /
// K3CUDA_ERR_TIMEOUT status instead of a hang: the reference's rule of never returning a
// result that was not computed (src/core/k3_ops.c:38-78), as a status this library can
// give. After an abort the context keeps working for single-GPU calls; its collective
// calls return K3CUDA_ERR_STATE.
#include <cuda.h>
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>
#include <time.h>

#include <vector>

#include "internal.cuh"

namespace k3 {

struct NcclApi {
    void *handle = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int,
                                       ncclConfig_t *) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                              ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi g_nccl;

static int nccl_load() {
    if (g_nccl.handle) return K3CUDA_OK;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return set_error(K3CUDA_ERR_NCCL, "cannot load libnccl.so.2: %s", dlerror());
#define K3_SYM(field, name)                                                              \
    g_nccl.field = (decltype(g_nccl.field))dlsym(h, name);                               \
    if (!g_nccl.field) return set_error(K3CUDA_ERR_NCCL, "libnccl lacks %s", name);
    K3_SYM(GetUniqueId, "ncclGetUniqueId");
    K3_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    K3_SYM(CommDestroy, "ncclCommDestroy");
    K3_SYM(CommAbort, "ncclCommAbort");
    K3_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    K3_SYM(AllGather, "ncclAllGather");
    K3_SYM(AllReduce, "ncclAllReduce");
    K3_SYM(GetErrorString, "ncclGetErrorString");
#undef K3_SYM
    g_nccl.handle = h;
    return K3CUDA_OK;
}

// full[t][r*Hl*dv + x] = gathered[r][t][x], moved in 16-byte units (Hl*dv*esize % 16 == 0).
__global__ void head_interleave(uint4 *__restrict__ full, const uint4 *__restrict__ gathered,
                                int T, int R, int row16) {
    const long long total = (long long)T * R * row16;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int x = (int)(e % row16);
        const long long tr = e / row16;
        const int r = (int)(tr % R);
        const long long t = tr / R;
        full[e] = gathered[((long long)r * T + t) * row16 + x];
    }
}

// Copy rows [t][head0 .. head0 + H_local) of this rank's full buffer into the same place of
// every peer's full buffer (peer memory over NVLink). Consecutive threads move consecutive
// 16-byte pieces of a token's contiguous head span, so each warp store is 512 B contiguous.
__global__ void push_heads(const uint4 *__restrict__ own, uint4 *const *__restrict__ peers,
                           int npeers, int T, long long row16, long long span16,
                           long long off16) {
    const long long total = (long long)T * span16;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long t = e / span16, x = e % span16;
        const long long at = t * row16 + off16 + x;
        const uint4 v = own[at];
        for (int r = 0; r < npeers; r++) peers[r][at] = v;
    }
}

int comm_push_heads(k3cuda_ctx *ctx, int T, int head0, int H_local, int H_total, int dv) {
    if (ctx->nranks <= 1 || T == 0) return K3CUDA_OK;
    uint4 *peers[K3CUDA_MAX_RANKS];
    int np = 0;
    for (int r = 0; r < ctx->nranks; r++)
        if (r != ctx->rank) peers[np++] = (uint4 *)ctx->full_out[r];
    if (!ctx->peer_table)
        K3_CUDA_TRY(cudaMalloc((void **)&ctx->peer_table, sizeof(void *) * K3CUDA_MAX_RANKS));
    K3_CUDA_TRY(cudaMemcpyAsync(ctx->peer_table, peers, sizeof(void *) * np,
                                cudaMemcpyHostToDevice, ctx->stream));
    const long long row16 = (long long)H_total * dv * 2 / 16;
    const long long span16 = (long long)H_local * dv * 2 / 16;
    const long long off16 = (long long)head0 * dv * 2 / 16;
    const long long total = (long long)T * span16;
    const int blocks = (int)((total + 255) / 256 < ctx->sm_count * 8 ? (total + 255) / 256
                                                                     : ctx->sm_count * 8);
    push_heads<<<blocks, 256, 0, ctx->stream>>>((const uint4 *)ctx->full_out[ctx->rank],
                                                (uint4 *const *)ctx->peer_table, np, T, row16,
                                                span16, off16);
    return after_launch(ctx, "push_heads");
}

static double now_ms() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

static void sleep_us(long us) {
    timespec ts{0, us * 1000};
    nanosleep(&ts, nullptr);
}

// Abort the communicator after a failure: pending collectives end, the stream drains, the
// peers' buffers are unmapped. Returns `code` with the message already set by the caller.
static int comm_abort(k3cuda_ctx *ctx, int code) {
    if (ctx->nccl_comm && g_nccl.handle) g_nccl.CommAbort((ncclComm_t)ctx->nccl_comm);
    ctx->nccl_comm = nullptr;
    ctx->comm_failed = 1;
    cudaStreamSynchronize(ctx->stream);
    cudaGetLastError();
    for (int r = 0; r < K3CUDA_MAX_RANKS; r++) {
        if (ctx->full_base[r]) cudaIpcCloseMemHandle(ctx->full_base[r]);
        ctx->full_base[r] = nullptr;
        ctx->full_out[r] = nullptr;
    }
    ctx->full_bytes = 0;
    return code;
}

// Wait until `done()` holds or the communicator reports a state other than in-progress /
// success, under the context's deadline. On failure the communicator is aborted.
template <typename Done>
static int comm_poll(k3cuda_ctx *ctx, const char *what, Done done) {
    const double t_end = now_ms() + ctx->comm_timeout_ms;
    for (long it = 0;; it++) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = g_nccl.CommGetAsyncError((ncclComm_t)ctx->nccl_comm, &st);
        if (r != ncclSuccess) st = r;
        if (st != ncclSuccess && st != ncclInProgress) {
            set_error(K3CUDA_ERR_NCCL, "%s: communicator failed: %s", what,
                      g_nccl.GetErrorString(st));
            return comm_abort(ctx, K3CUDA_ERR_NCCL);
        }
        if (st == ncclSuccess && done()) return K3CUDA_OK;
        if (now_ms() > t_end) {
            set_error(K3CUDA_ERR_TIMEOUT,
                      "%s: no progress within %d ms (a peer left or stalled); communicator "
                      "aborted", what, ctx->comm_timeout_ms);
            return comm_abort(ctx, K3CUDA_ERR_TIMEOUT);
        }
        sleep_us(it < 100 ? 5 : 200);
    }
}

// A non-blocking communicator may return ncclInProgress from an enqueue: it is complete
// once the asynchronous state reads success again.
static int comm_enqueued(k3cuda_ctx *ctx, ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return K3CUDA_OK;
    if (r == ncclInProgress) return comm_poll(ctx, what, [] { return true; });
    set_error(K3CUDA_ERR_NCCL, "%s: %s", what, g_nccl.GetErrorString(r));
    return comm_abort(ctx, K3CUDA_ERR_NCCL);
}

int comm_wait_stream(k3cuda_ctx *ctx) {
    if (!ctx->nccl_comm) return K3CUDA_OK;
    return comm_poll(ctx, "k3cuda_sync", [ctx] {
        return cudaStreamQuery(ctx->stream) != cudaErrorNotReady;
    });
}

static int comm_usable(k3cuda_ctx *ctx) {
    if (ctx->comm_failed)
        return set_error(K3CUDA_ERR_STATE, "the communicator was aborted after a failure");
    if (!ctx->nccl_comm) return set_error(K3CUDA_ERR_STATE, "k3cuda_comm_init not called");
    return K3CUDA_OK;
}

// Stream-ordered fence across the ranks: a one-int all-reduce completes on every rank only
// after every rank has reached it (so all work enqueued before it, on every rank, is done).
// wait_host: the host also waits for it under the deadline, so that nothing enqueued after
// it (peer stores) can run once a peer has gone.
int comm_fence(k3cuda_ctx *ctx, bool wait_host) {
    if (ctx->nranks <= 1) return K3CUDA_OK;
    int rc = comm_enqueued(ctx,
                           g_nccl.AllReduce(ctx->sync_word, ctx->sync_word, 1, ncclInt32,
                                            ncclSum, (ncclComm_t)ctx->nccl_comm, ctx->stream),
                           "fence (ncclAllReduce)");
    if (rc || !wait_host) return rc;
    K3_CUDA_TRY(cudaEventRecord(ctx->ev_fence, ctx->stream));
    return comm_poll(ctx, "fence", [ctx] {
        return cudaEventQuery(ctx->ev_fence) != cudaErrorNotReady;
    });
}

}  // namespace k3

using namespace k3;

extern "C" {

int k3cuda_comm_destroy_internal(k3cuda_ctx *ctx) {
    if (!ctx) return K3CUDA_OK;
    for (int r = 0; r < K3CUDA_MAX_RANKS; r++) {
        if (ctx->full_base[r]) cudaIpcCloseMemHandle(ctx->full_base[r]);
        ctx->full_out[r] = nullptr;
        ctx->full_base[r] = nullptr;
    }
    if (ctx->sync_word) cudaFree(ctx->sync_word);
    ctx->sync_word = nullptr;
    if (ctx->peer_table) cudaFree(ctx->peer_table);
    ctx->peer_table = nullptr;
    if (ctx->nccl_comm && g_nccl.handle) {
        g_nccl.CommDestroy((ncclComm_t)ctx->nccl_comm);
        ctx->nccl_comm = nullptr;
    }
    return K3CUDA_OK;
}

int k3cuda_comm_unique_id(unsigned char id[K3CUDA_UNIQUE_ID_BYTES]) {
    K3_ARG_CHECK(id, "null id buffer");
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId uid;
    ncclResult_t r = g_nccl.GetUniqueId(&uid);
    if (r != ncclSuccess)
        return set_error(K3CUDA_ERR_NCCL, "ncclGetUniqueId: %s", g_nccl.GetErrorString(r));
    static_assert(sizeof(uid) == K3CUDA_UNIQUE_ID_BYTES, "unique id size");
    memcpy(id, &uid, sizeof uid);
    return K3CUDA_OK;
}

int k3cuda_comm_init(k3cuda_ctx *ctx, int nranks, int rank,
                     const unsigned char id[K3CUDA_UNIQUE_ID_BYTES]) {
    int rc = enter(ctx);
    if (rc) return rc;
    K3_ARG_CHECK(id && nranks >= 1 && rank >= 0 && rank < nranks, "bad comm_init arguments");
    rc = nccl_load();
    if (rc) return rc;
    if (ctx->nccl_comm || ctx->comm_failed)
        return set_error(K3CUDA_ERR_STATE, "communicator already initialised");
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclComm_t comm = nullptr;
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every host wait is ours, under a deadline
    ncclResult_t r = g_nccl.CommInitRankConfig(&comm, nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (comm) g_nccl.CommAbort(comm);
        return set_error(K3CUDA_ERR_NCCL, "ncclCommInitRankConfig: %s", g_nccl.GetErrorString(r));
    }
    ctx->nccl_comm = comm;
    ctx->nranks = nranks;
    ctx->rank = rank;
    rc = comm_poll(ctx, "ncclCommInitRankConfig", [] { return true; });
    if (rc) {
        ctx->nranks = 1;
        ctx->rank = 0;
    }
    return rc;
}

int k3cuda_comm_set_timeout(k3cuda_ctx *ctx, int ms) {
    K3_ARG_CHECK(ctx && ms > 0, "bad communicator timeout");
    ctx->comm_timeout_ms = ms;
    return K3CUDA_OK;
}

int k3cuda_comm_register_full(k3cuda_ctx *ctx, void *full, size_t bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    if ((rc = comm_usable(ctx))) return rc;
    K3_ARG_CHECK(full && bytes && aligned(full, 16), "register_full: bad buffer");
    K3_ARG_CHECK(ctx->nranks <= K3CUDA_MAX_RANKS, "register_full: at most %d ranks",
                 K3CUDA_MAX_RANKS);
    if (ctx->full_out[ctx->rank])
        return set_error(K3CUDA_ERR_STATE, "register_full: a buffer is already registered");
    // this rank's record: IPC handle of the allocation holding `full`, offset of `full` in it
    struct Rec {
        cudaIpcMemHandle_t h;
        unsigned long long off, bytes;
    };
    static_assert(sizeof(Rec) % 16 == 0, "record size");
    Rec mine{};
    if (ctx->nranks > 1) {
        void *base = nullptr;
        size_t range = 0;
        CUdeviceptr b = 0;
        // allocation base through the driver entry point (no libcuda link)
        static CUresult (*get_range)(CUdeviceptr *, size_t *, CUdeviceptr) = nullptr;
        if (!get_range) {
            void *fp = nullptr;
            cudaDriverEntryPointQueryResult qr;
            if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fp, cudaEnableDefault, &qr) !=
                    cudaSuccess ||
                qr != cudaDriverEntryPointSuccess)
                return set_error(K3CUDA_ERR_CUDA, "cuMemGetAddressRange unavailable");
            get_range = (CUresult(*)(CUdeviceptr *, size_t *, CUdeviceptr))fp;
        }
        if (get_range(&b, &range, (CUdeviceptr)full) != CUDA_SUCCESS)
            return set_error(K3CUDA_ERR_ARG, "register_full: not device memory");
        base = (void *)b;
        K3_CUDA_TRY(cudaIpcGetMemHandle(&mine.h, base));
        mine.off = (unsigned long long)((char *)full - (char *)base);
    }
    mine.bytes = bytes;
    std::vector<Rec> all(ctx->nranks);
    if (ctx->nranks > 1) {
        // exchange the records with one all-gather through a temporary device buffer that
        // every path below frees
        Rec *d = nullptr;
        cudaError_t e = cudaMalloc((void **)&d, sizeof(Rec) * (ctx->nranks + 1));
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d + ctx->nranks, &mine, sizeof mine, cudaMemcpyHostToDevice,
                                ctx->stream);
        if (e != cudaSuccess) {
            if (d) cudaFree(d);
            return set_error(K3CUDA_ERR_CUDA, "register_full: %s", cudaGetErrorString(e));
        }
        rc = comm_enqueued(ctx,
                           g_nccl.AllGather(d + ctx->nranks, d, sizeof(Rec), ncclUint8,
                                            (ncclComm_t)ctx->nccl_comm, ctx->stream),
                           "register_full (ncclAllGather)");
        if (!rc) {
            e = cudaMemcpyAsync(all.data(), d, sizeof(Rec) * ctx->nranks, cudaMemcpyDeviceToHost,
                                ctx->stream);
            if (e != cudaSuccess)
                rc = set_error(K3CUDA_ERR_CUDA, "register_full: %s", cudaGetErrorString(e));
        }
        if (!rc) rc = comm_wait_stream(ctx);
        if (!rc) {
            e = cudaStreamSynchronize(ctx->stream);
            if (e != cudaSuccess)
                rc = set_error(K3CUDA_ERR_CUDA, "register_full: %s", cudaGetErrorString(e));
        }
        cudaFree(d);
        if (rc) return rc;
    } else {
        all[0] = mine;
    }
    size_t common = bytes;
    for (int r = 0; r < ctx->nranks; r++) common = all[r].bytes < common ? all[r].bytes : common;
    for (int r = 0; r < ctx->nranks; r++) {
        if (r == ctx->rank) continue;
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, all[r].h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            // undo the mappings made so far, so that a later attempt starts clean
            for (int q = 0; q < r; q++) {
                if (ctx->full_base[q]) cudaIpcCloseMemHandle(ctx->full_base[q]);
                ctx->full_base[q] = nullptr;
                ctx->full_out[q] = nullptr;
            }
            return set_error(K3CUDA_ERR_CUDA, "register_full: opening rank %d's buffer: %s", r,
                             cudaGetErrorString(e));
        }
        ctx->full_base[r] = p;
        ctx->full_out[r] = (char *)p + all[r].off;
    }
    if (!ctx->sync_word) {
        cudaError_t e = cudaMalloc((void **)&ctx->sync_word, sizeof(int));
        if (e != cudaSuccess) {
            for (int q = 0; q < ctx->nranks; q++) {
                if (ctx->full_base[q]) cudaIpcCloseMemHandle(ctx->full_base[q]);
                ctx->full_base[q] = nullptr;
                ctx->full_out[q] = nullptr;
            }
            return set_error(K3CUDA_ERR_CUDA, "register_full: %s", cudaGetErrorString(e));
        }
    }
    ctx->full_out[ctx->rank] = full;
    ctx->full_bytes = common;
    return K3CUDA_OK;
}

int k3cuda_allgather_heads_workspace(int nranks, int T, int H_local, int dv, int dtype,
                                     size_t *bytes) {
    K3_ARG_CHECK(bytes && nranks >= 1 && T >= 0 && H_local >= 1 && dv >= 1, "bad arguments");
    K3_ARG_CHECK(dtype == K3CUDA_F32 || dtype == K3CUDA_BF16, "bad dtype");
    const size_t es = dtype == K3CUDA_BF16 ? 2 : 4;
    *bytes = (size_t)nranks * T * H_local * dv * es;
    return K3CUDA_OK;
}

int k3cuda_allgather_heads(k3cuda_ctx *ctx, void *full, const void *local, int T, int H_local,
                           int dv, int dtype, void *workspace, size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    if ((rc = comm_usable(ctx))) return rc;
    size_t need = 0;
    rc = k3cuda_allgather_heads_workspace(ctx->nranks, T, H_local, dv, dtype, &need);
    if (rc) return rc;
    if (T == 0) return K3CUDA_OK;
    K3_ARG_CHECK(full && local, "null pointer");
    if (workspace_bytes < need || !workspace)
        return set_error(K3CUDA_ERR_WORKSPACE, "allgather: workspace %zu < %zu", workspace_bytes,
                         need);
    const size_t es = dtype == K3CUDA_BF16 ? 2 : 4;
    const size_t row = (size_t)H_local * dv * es;
    if (row % 16 || !aligned(full, 16) || !aligned(workspace, 16))
        return set_error(K3CUDA_ERR_ARG, "allgather: rows must be 16-byte multiples and aligned");
    const size_t count = (size_t)T * H_local * dv;
    rc = comm_enqueued(ctx,
                       g_nccl.AllGather(local, workspace, count,
                                        dtype == K3CUDA_BF16 ? ncclBfloat16 : ncclFloat32,
                                        (ncclComm_t)ctx->nccl_comm, ctx->stream),
                       "ncclAllGather");
    if (rc) return rc;
    const int row16 = (int)(row / 16);
    const long long total = (long long)T * ctx->nranks * row16;
    const int blocks = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    head_interleave<<<blocks, 256, 0, ctx->stream>>>((uint4 *)full, (const uint4 *)workspace, T,
                                                     ctx->nranks, row16);
    return after_launch(ctx, "head_interleave");
}

}  // extern "C"
