// noalloc_gw.cu -- group-wise int4 matmul for callers that cannot allocate.
//
// Some callers may not call cudaMalloc at all: an inference runtime that owns
// every byte of device memory through its own arena, a process whose memory
// budget is fixed up front, or a host that must not allocate while it runs
// (a real-time or safety-certified loop).  rocket_matmul_int4_groupwise needs
// device scratch and takes it from a per-handle pool that grows with
// cudaMalloc.  This file computes the library's fast group-wise form (the one
// rocket_b200_gw_mode(1) selects: w * b_scale rounded to fp16 before an fp16
// MMA, about 3e-4 relative error), whose scratch -- the packed nibble codes,
// the packed fp16 scales and the pre-scaled fp16 activations -- sits in one
// fixed array compiled into the library, so nothing is allocated per call.
//
// Cost of the array: RKB_NOALLOC_SCRATCH_BYTES (32 MiB) of device memory on
// every GPU that loads this library, held until the process exits.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../src/rkb_kernels.h"
#include "../../include/rocket_npu.h"
#include "../../include/rocket_log.h"
#include "../../include/rocket_b200.h"

#define RKB_NOALLOC_SCRATCH_BYTES (32u << 20)
#define RKB_NOALLOC_MAX_DEVICES 64

// Shared by every call on a device; keeps whatever the last call left in it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[RKB_NOALLOC_SCRATCH_BYTES];

namespace {

// Device address of g_noalloc_scratch per device.  In host code the array's
// name is only a host-side stand-in; the real address comes from
// cudaGetSymbolAddress with the device current, once per device.
unsigned char *g_scratch_addr[RKB_NOALLOC_MAX_DEVICES];

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

bool is_device_ptr_on(const void *p, int dev) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.device == dev;
}

}  // namespace

extern "C" int rocket_b200_matmul_int4_groupwise_noalloc(int M, int K, int N, const int8_t *A,
                                                          const int8_t *B, const float *a_scale,
                                                          const float *b_scale, float *Cf, int group,
                                                          void *stream) {
    const char *who = "rocket_b200_matmul_int4_groupwise_noalloc";
    if (M <= 0 || M % 4 || K <= 0 || K % 32 || N <= 0 || N % 64 || group < 32 || group % 32 ||
        K % group || 49 * group >= 32767 || !A || !B || !a_scale || !b_scale || !Cf) {
        rocket_log(ROCKET_LOG_ERROR, "%s: bad shape M=%d K=%d N=%d group=%d\n", who, M, K, N, group);
        return ROCKET_E_SHAPE;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= RKB_NOALLOC_MAX_DEVICES) {
        cudaGetLastError();
        return ROCKET_E_DEVICE;
    }
    // Scratch layout: error word | packed codes | packed scales | fp16 A.
    const size_t off_codes = 256;
    const size_t off_scales = off_codes + align256(rkb_wpack_codes_bytes(N, K, 4));
    const size_t off_a = off_scales + align256(rkb_wpack_scales_bytes(N, K));
    const size_t need = off_a + align256(static_cast<size_t>(M) * K * 2);
    if (need > RKB_NOALLOC_SCRATCH_BYTES) {
        rocket_log(ROCKET_LOG_ERROR,
                   "%s: M=%d K=%d N=%d needs %zu bytes of scratch, above the fixed %u-byte array\n",
                   who, M, K, N, need, RKB_NOALLOC_SCRATCH_BYTES);
        return ROCKET_E_NOMEM;
    }
    if (!is_device_ptr_on(A, dev) || !is_device_ptr_on(B, dev) || !is_device_ptr_on(a_scale, dev) ||
        !is_device_ptr_on(b_scale, dev) || !is_device_ptr_on(Cf, dev) ||
        (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(Cf) & 15)) {
        rocket_log(ROCKET_LOG_ERROR,
                   "%s: A, B, a_scale, b_scale and Cf must be device memory on the current GPU "
                   "(A and Cf 16-byte aligned); this entry copies nothing\n", who);
        return ROCKET_E_SHAPE;
    }
    // One-time set-up on this device (see the header: make the first call
    // outside any stream capture).
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            rocket_log(ROCKET_LOG_ERROR, "%s: cudaGetSymbolAddress failed: %s\n", who,
                       cudaGetErrorString(e));
            cudaGetLastError();
            return ROCKET_E_DEVICE;
        }
        g_scratch_addr[dev] = static_cast<unsigned char *>(p);
    }
    unsigned char *base = g_scratch_addr[dev];
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int *err = reinterpret_cast<int *>(base);
    void *codes = base + off_codes;
    void *scales = base + off_scales;
    void *af = base + off_a;

    // The error word must start at zero; everything else is fully rewritten.
    int rc = cudaMemsetAsync(err, 0, sizeof(int), s) == cudaSuccess ? 0 : ROCKET_E_DEVICE;
    if (!rc) rc = rkb_wpack_codes(B, N, K, 4, codes, s);
    if (!rc) rc = rkb_wpack_scales(b_scale, N, K, group, scales, s);
    if (!rc) rc = rkb_prescale_a(A, a_scale, M, K, group, af, s);
    if (!rc) {
        rkb_wgemm_desc d;
        memset(&d, 0, sizeof d);
        d.M = M; d.N = N; d.K = K; d.w_bits = 4; d.a_f16 = 1;
        d.A = af; d.lda = K; d.Wq = codes; d.Ws = scales;
        d.C = Cf; d.ldc = N; d.out_kind = RKB_OUT_F32; d.row_scale = nullptr;
        rc = rkb_wgemm_run(&d, err, s);
    }
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        rocket_log(ROCKET_LOG_ERROR, "%s: CUDA error: %s\n", who, cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    if (rc) return rc;
    int ew = 0;
    if (cudaMemcpy(&ew, err, sizeof ew, cudaMemcpyDeviceToHost) != cudaSuccess) return ROCKET_E_DEVICE;
    if (ew) {
        rocket_log(ROCKET_LOG_ERROR, "%s: kernel pipeline wait expired (code %d)\n", who, ew);
        return ROCKET_E_DEVICE;
    }
    return 0;
}
