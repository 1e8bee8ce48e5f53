// Host-side TMA tensor-map encoding through the runtime's driver entry point, so the
// library loads (and its CPU-only tests run) without libcuda being present.
#include "kernels.h"

#include <cudaTypedefs.h>

#include <mutex>
#include <string>

namespace hyb {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        HYB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p) throw CudaError("cuTensorMapEncodeTiled is not available");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}
}  // namespace

void encode_tma(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
    if (reinterpret_cast<uintptr_t>(base) & 15) throw ArgError("tensor map base must be 16-byte aligned");
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) {
            if (strides_bytes[i] % 16 != 0) throw ArgError("tensor map strides must be multiples of 16 bytes");
            st[i] = strides_bytes[i];
        }
    }
    const CUresult r = encode_fn()(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st, b, es,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r)));
}

}  // namespace hyb
