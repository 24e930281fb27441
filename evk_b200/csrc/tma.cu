// tma.cu — host-side TMA tensor-map encoding through the driver entry point.
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "sm100.cuh"

namespace evkcu {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_elems,
                 uint64_t stride2_elems, uint32_t box0, uint32_t box1, int dtype, bool swizzle128) {
    auto fn = encode_fn();
    if (!fn) return fail(EVKCU_CUDA_ERROR, "cuTensorMapEncodeTiled entry point unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(EVKCU_BAD_ALIGN, "TMA base not 16-byte aligned");
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {stride1_elems * 2, stride2_elems * 2};
    if ((strides[0] & 15u) || (strides[1] & 15u))
        return fail(EVKCU_BAD_ALIGN, "TMA row/batch pitch must be a multiple of 16 bytes (8 elements)");
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estride[3] = {1, 1, 1};
    CUtensorMapDataType dt = dtype == EVKCU_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(EVKCU_BAD_SHAPE, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
    return EVKCU_OK;
}

}  // namespace evkcu
