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

// Per-thread cache of encoded tensor maps: encoding costs about a microsecond of
// host time, which matters for short GEMMs issued back to back on the same
// buffers.  Keyed on every argument of the encode.
struct TmapKey {
    const void *base;
    long cols, rows, ld;
    int dt, esize, box_cols, box_rows, swz;
    bool operator==(const TmapKey &o) const {
        return base == o.base && cols == o.cols && rows == o.rows && ld == o.ld && dt == o.dt &&
               esize == o.esize && box_cols == o.box_cols && box_rows == o.box_rows && swz == o.swz;
    }
};

// Row-major 2D tensor [rows, cols] (cols contiguous, ld elements between rows),
// box = box_cols x box_rows, 128-byte swizzle, zero fill outside the tensor.
// Returns 0 on success.  box_cols * esize must be <= 128 for the swizzle and
// the base / row pitch must be 16-byte aligned.
inline int encode_tmap_2d(CUtensorMap *tm, const void *base, CUtensorMapDataType dt, int esize,
                          long cols, long rows, long ld, int box_cols, int box_rows,
                          CUtensorMapSwizzle swz) {
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

// Row-major 3D tensor [planes, rows, cols] (plane pitch and row pitch in
// elements), box box_cols x box_rows x 1.  Not cached (split-K partial slabs only).
inline int encode_tmap_3d(CUtensorMap *tm, const void *base, CUtensorMapDataType dt, int esize, long cols,
                          long rows, long planes, long ld, long plane_ld, int box_cols, int box_rows,
                          CUtensorMapSwizzle swz) {
    auto enc = tmap_encoder();
    if (!enc) return -1;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * esize) & 15) || ((plane_ld * esize) & 15)) return -1;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(planes)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * esize, static_cast<cuuint64_t>(plane_ld) * esize};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(tm, dt, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -1;
}

inline int make_tmap_2d(CUtensorMap *tm, const void *base, CUtensorMapDataType dt, int esize,
                        long cols, long rows, long ld, int box_cols, int box_rows,
                        CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    constexpr int SLOTS = 64;
    static thread_local TmapKey keys[SLOTS];
    static thread_local CUtensorMap maps[SLOTS];
    static thread_local bool valid[SLOTS];
    const TmapKey k{base, cols, rows, ld, static_cast<int>(dt), esize, box_cols, box_rows, static_cast<int>(swz)};
    const size_t h = (reinterpret_cast<uintptr_t>(base) >> 8) ^ static_cast<size_t>(cols * 31 + rows * 17 + box_rows);
    const int slot = static_cast<int>(h % SLOTS);
    if (valid[slot] && keys[slot] == k) {
        *tm = maps[slot];
        return 0;
    }
    int rc = encode_tmap_2d(tm, base, dt, esize, cols, rows, ld, box_cols, box_rows, swz);
    if (rc == 0) {
        keys[slot] = k;
        maps[slot] = *tm;
        valid[slot] = true;
    }
    return rc;
}

}  // namespace rkb
