// tmap.cu -- TMA tensor-map encoding through the driver entry point (no libcuda link).
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "ane_internal.cuh"

namespace ane_b200 {

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        set_status(ANE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
        return ANE_ERR_CUDA;
    }
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_status(ANE_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
        return ANE_ERR_CUDA;
    }
    return ANE_OK;
}

int encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t (&dims)[3],
                         const uint64_t (&stride_bytes)[2], const uint32_t (&box)[3]) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        set_status(ANE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
        return ANE_ERR_CUDA;
    }
    cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    cuuint64_t st[2] = {stride_bytes[0], stride_bytes[1]};
    cuuint32_t bx[3] = {box[0], box[1], box[2]};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, dtype, 3, const_cast<void*>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_status(ANE_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed: " + std::to_string((int)r));
        return ANE_ERR_CUDA;
    }
    return ANE_OK;
}

}  // namespace ane_b200
