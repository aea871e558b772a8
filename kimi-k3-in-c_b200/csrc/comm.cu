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
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include "internal.cuh"

namespace k3 {

struct NcclApi {
    void *handle = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
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
    K3_SYM(CommInitRank, "ncclCommInitRank");
    K3_SYM(CommDestroy, "ncclCommDestroy");
    K3_SYM(CommAbort, "ncclCommAbort");
    K3_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    K3_SYM(AllGather, "ncclAllGather");
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

}  // namespace k3

using namespace k3;

extern "C" {

int k3cuda_comm_destroy_internal(k3cuda_ctx *ctx) {
    if (ctx && ctx->nccl_comm && g_nccl.handle) {
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
    if (ctx->nccl_comm) return set_error(K3CUDA_ERR_STATE, "communicator already initialised");
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclComm_t comm = nullptr;
    ncclResult_t r = g_nccl.CommInitRank(&comm, nranks, uid, rank);
    if (r != ncclSuccess)
        return set_error(K3CUDA_ERR_NCCL, "ncclCommInitRank: %s", g_nccl.GetErrorString(r));
    ctx->nccl_comm = comm;
    ctx->nranks = nranks;
    ctx->rank = rank;
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
    if (!ctx->nccl_comm) return set_error(K3CUDA_ERR_STATE, "k3cuda_comm_init not called");
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
    ncclResult_t r = g_nccl.AllGather(local, workspace, count,
                                      dtype == K3CUDA_BF16 ? ncclBfloat16 : ncclFloat32,
                                      (ncclComm_t)ctx->nccl_comm, ctx->stream);
    if (r != ncclSuccess)
        return set_error(K3CUDA_ERR_NCCL, "ncclAllGather: %s", g_nccl.GetErrorString(r));
    const int row16 = (int)(row / 16);
    const long long total = (long long)T * ctx->nranks * row16;
    const int blocks = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    head_interleave<<<blocks, 256, 0, ctx->stream>>>((uint4 *)full, (const uint4 *)workspace, T,
                                                     ctx->nranks, row16);
    return after_launch(ctx, "head_interleave");
}

}  // extern "C"
