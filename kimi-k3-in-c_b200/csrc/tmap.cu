// tmap.cu -- TMA tensor-map creation through the driver entry point (see tmap.cuh).
#include <cudaTypedefs.h>

#include "internal.cuh"
#include "tmap.cuh"

namespace k3 {

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
    return K3CUDA_OK;
}

int make_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype,
                 uint32_t elem_bytes, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                 uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2) {
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
    return K3CUDA_OK;
}

}  // namespace k3
