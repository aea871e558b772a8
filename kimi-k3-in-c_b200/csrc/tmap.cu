// tmap.cu -- TMA tensor-map creation through the driver entry point (see tmap.cuh).
#include <cudaTypedefs.h>
#include <string.h>

#include <mutex>

#include "internal.cuh"
#include "tmap.cuh"

namespace k3 {

// Encoded maps are cached by their full description (address, type, sizes, strides, box):
// a map is a pure function of those, and the driver's encode call costs microseconds of host
// time that a decode step repeats for the same tensors every call.
struct TmapKey {
    const void *base;
    uint64_t dims[3], strides[2];
    uint32_t rank, dtype, elem, box[3];
};
struct TmapEntry {
    TmapKey key;
    CUtensorMap map;
    bool used;
};
constexpr int TMAP_CACHE = 256;
static TmapEntry g_tmaps[TMAP_CACHE];
static int g_tmap_next = 0;
static std::mutex g_tmap_mu;

static bool tmap_lookup(const TmapKey &k, CUtensorMap *map) {
    std::lock_guard<std::mutex> lk(g_tmap_mu);
    for (int i = 0; i < TMAP_CACHE; i++)
        if (g_tmaps[i].used && memcmp(&g_tmaps[i].key, &k, sizeof k) == 0) {
            *map = g_tmaps[i].map;
            return true;
        }
    return false;
}

static void tmap_store(const TmapKey &k, const CUtensorMap &map) {
    std::lock_guard<std::mutex> lk(g_tmap_mu);
    TmapEntry &e = g_tmaps[g_tmap_next];
    g_tmap_next = (g_tmap_next + 1) % TMAP_CACHE;
    e.key = k;
    e.map = map;
    e.used = true;
}

static TmapKey tmap_key(uint32_t rank, const void *base, CUtensorMapDataType dtype, uint32_t elem,
                        const uint64_t *dims, const uint64_t *strides, const uint32_t *box) {
    TmapKey k;
    memset(&k, 0, sizeof k);  // padding bytes take part in the comparison
    k.base = base;
    k.rank = rank;
    k.dtype = (uint32_t)dtype;
    k.elem = elem;
    for (uint32_t i = 0; i < rank; i++) {
        k.dims[i] = dims[i];
        k.box[i] = box[i];
    }
    for (uint32_t i = 0; i + 1 < rank; i++) k.strides[i] = strides[i];
    return k;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

int make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype,
                 uint32_t elem_bytes, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer) {
    const uint64_t kd[2] = {inner, outer}, ks[1] = {row_bytes};
    const uint32_t kb[2] = {box_inner, box_outer};
    const TmapKey key = tmap_key(2, base, dtype, elem_bytes, kd, ks, kb);
    if (tmap_lookup(key, map)) return K3CUDA_OK;
    auto fn = encode_fn();
    if (!fn) return set_error(K3CUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = box_inner * elem_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(K3CUDA_ERR_CUDA, "cuTensorMapEncodeTiled(2d) failed: %d", (int)r);
    tmap_store(key, *map);
    return K3CUDA_OK;
}

int make_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype,
                 uint32_t elem_bytes, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                 uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2) {
    const uint64_t kd[3] = {d0, d1, d2}, ks[2] = {s1, s2};
    const uint32_t kb[3] = {b0, b1, b2};
    const TmapKey key = tmap_key(3, base, dtype, elem_bytes, kd, ks, kb);
    if (tmap_lookup(key, map)) return K3CUDA_OK;
    auto fn = encode_fn();
    if (!fn) return set_error(K3CUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle sw =
        b0 * elem_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = fn(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(K3CUDA_ERR_CUDA, "cuTensorMapEncodeTiled(3d) failed: %d", (int)r);
    tmap_store(key, *map);
    return K3CUDA_OK;
}

}  // namespace k3
