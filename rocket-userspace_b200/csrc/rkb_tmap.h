// rkb_tmap.h -- building TMA tensor maps without linking libcuda: the driver's
// cuTensorMapEncodeTiled is fetched once through cudaGetDriverEntryPoint.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>

namespace rkb {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Row-major 2D tensor [rows, cols] (cols contiguous, ld elements between rows),
// box = box_cols x box_rows, 128-byte swizzle, zero fill outside the tensor.
// Returns 0 on success.  box_cols * esize must be <= 128 for the swizzle and
// the base / row pitch must be 16-byte aligned.
inline int make_tmap_2d(CUtensorMap *tm, const void *base, CUtensorMapDataType dt, int esize,
                        long cols, long rows, long ld, int box_cols, int box_rows,
                        CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    auto enc = tmap_encoder();
    if (!enc) {
        fprintf(stderr, "rkb: cuTensorMapEncodeTiled unavailable\n");
        return -1;
    }
    if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * esize) & 15)) return -1;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esize};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fprintf(stderr, "rkb: cuTensorMapEncodeTiled failed (%d) cols=%ld rows=%ld ld=%ld\n",
                static_cast<int>(r), cols, rows, ld);
        return -1;
    }
    return 0;
}

}  // namespace rkb
