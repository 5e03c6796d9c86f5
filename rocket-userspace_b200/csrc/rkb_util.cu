// rkb_util.cu -- small HBM-bound helper kernels around the GEMMs: the resident
// weight packers (row-major int8 [N,K] -> tiled offset-binary code blocks and
// fp16 scale blocks), activation pre-scaling for group-wise A scales, and a
// per-device SM-count cache.  All are one pass over their input with
// coalesced loads; none is on the timed path of a prepacked call except
// rkb_prescale_a (M*K bytes in, 2*M*K bytes out).
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include "../src/rkb_kernels.h"
#include "rkb_wlayout.cuh"
#include "../../include/rocket_npu.h"

namespace {

// dst byte i -> (tile t, block kb, row r, byte j) of the ragged tiled layout
// (rkb_wlayout.cuh); rb = bytes per row of one 64-wide K block
__device__ __forceinline__ void wl_decode(size_t i, int N, int nkb, int rb, int &n, int &kb, int &j) {
    const size_t tile_bytes = static_cast<size_t>(nkb) * rkb::WL_TILE * rb;
    int t = static_cast<int>(i / tile_bytes);
    const int last = rkb::wl_ntiles(N) - 1;
    t = t > last ? last : t;
    const size_t local = i - static_cast<size_t>(t) * tile_bytes;
    const size_t blk = static_cast<size_t>(rkb::wl_rows(N, t)) * rb;
    kb = static_cast<int>(local / blk);
    const int rem = static_cast<int>(local % blk);
    n = t * rkb::WL_TILE + rem / rb;
    j = rem % rb;
}

__global__ void pack_codes_i8(const int8_t *__restrict__ src, int N, int K, int nkb,
                              uint8_t *__restrict__ dst, size_t total) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        int n, kb, j;
        wl_decode(i, N, nkb, 64, n, kb, j);
        const int k = kb * 64 + j;
        int8_t v = (n < N && k < K) ? src[static_cast<size_t>(n) * K + k] : 0;
        dst[i] = static_cast<uint8_t>(v) ^ 0x80u;
    }
}

__global__ void pack_codes_i4(const int8_t *__restrict__ src, int N, int K, int nkb,
                              uint8_t *__restrict__ dst, size_t total) {
    // rows of 32 bytes; byte j holds codes 2j (low nibble) and 2j+1 (high)
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        int n, kb, j;
        wl_decode(i, N, nkb, 32, n, kb, j);
        const int k = kb * 64 + 2 * j;
        int v0 = 0, v1 = 0;
        if (n < N) {
            const int8_t *row = src + static_cast<size_t>(n) * K;
            if (k < K) v0 = row[k];
            if (k + 1 < K) v1 = row[k + 1];
        }
        dst[i] = static_cast<uint8_t>(((v0 + 8) & 15) | (((v1 + 8) & 15) << 4));
    }
}

// Tiled fp16 scales, rows of 2 halves (one per 32-wide K half of a block) in
// the same ragged layout: one thread per weight row of a tile, 16 K-blocks
// per CUDA block; each row's pair goes out as one 32-bit word.  bs == nullptr
// writes 1.0.
__global__ void pack_scales(const float *__restrict__ bs, int N, int K, int group, int nkb,
                            uint32_t *__restrict__ dst) {
    const int r = threadIdx.x;                 // blockDim.x == WL_TILE
    const int nt = blockIdx.y;
    const int rows = rkb::wl_rows(N, nt);
    if (r >= rows) return;
    const int n = nt * rkb::WL_TILE + r;
    const int nG = K / group;
    const int kb0 = blockIdx.x * 16;
    const int kb1 = kb0 + 16 < nkb ? kb0 + 16 : nkb;
    for (int kb = kb0; kb < kb1; ++kb) {
        float s0 = 1.0f, s1 = 1.0f;
        if (bs) {
            const int k0 = kb * 64, k1 = kb * 64 + 32;
            s0 = (n < N && k0 < K) ? bs[static_cast<size_t>(n) * nG + k0 / group] : 0.0f;
            s1 = (n < N && k1 < K) ? bs[static_cast<size_t>(n) * nG + k1 / group] : 0.0f;
        }
        __half2 h = __floats2half2_rn(s0, s1);
        dst[rkb::wl_block(N, nkb, nt, kb, 4) / 4 + r] = *reinterpret_cast<uint32_t *>(&h);
    }
}

// A16[m, k] = A[m, k] * a_scale[m, k / group] (or A[m, k] when as == nullptr).
// Grid (ceil(K / 4096), rows); 16 elements per thread.  K % 16 == 0.  VEC: A
// and dst 16-byte aligned (vector loads / stores), else byte loads.
template <bool VEC>
__global__ void prescale_a(const int8_t *__restrict__ A, const float *__restrict__ as, int M,
                           int K, int group, __half *__restrict__ dst) {
    const int k = (blockIdx.x * blockDim.x + threadIdx.x) * 16;
    if (k >= K) return;
    const int nG = as ? K / group : 0;
    for (int m = blockIdx.y; m < M; m += gridDim.y) {
        const size_t e = static_cast<size_t>(m) * K + k;
        int8_t b[16];
        if (VEC) {
            *reinterpret_cast<uint4 *>(b) = *reinterpret_cast<const uint4 *>(A + e);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) b[j] = A[e + j];
        }
        const float *srow = as ? as + static_cast<size_t>(m) * nG : nullptr;
        const bool one = (group % 16) == 0;   // all 16 elements in one group
        const float s_all = srow ? srow[k / group] : 1.0f;
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float s0 = (srow && !one) ? srow[(k + 2 * j) / group] : s_all;
            const float s1 = (srow && !one) ? srow[(k + 2 * j + 1) / group] : s_all;
            __half2 p = __floats2half2_rn(static_cast<float>(b[2 * j]) * s0, static_cast<float>(b[2 * j + 1]) * s1);
            o[j] = *reinterpret_cast<uint32_t *>(&p);
        }
        if (VEC) {
            uint4 *d = reinterpret_cast<uint4 *>(dst + e);
            d[0] = make_uint4(o[0], o[1], o[2], o[3]);
            d[1] = make_uint4(o[4], o[5], o[6], o[7]);
        } else {
            uint32_t *d = reinterpret_cast<uint32_t *>(dst + e);   // dst 4-byte aligned, K even
#pragma unroll
            for (int j = 0; j < 8; ++j) d[j] = o[j];
        }
    }
}

__global__ void gather_row_scale(const float *__restrict__ as, int M, int nG, float *__restrict__ dst) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m < M) dst[m] = as[static_cast<size_t>(m) * nG];
}

// a_scale [M, nG] -> [nG, M]: the precise group-wise epilogue reads one
// group's activation scales for 32 consecutive tokens with one load per lane
__global__ void scale_transpose(const float *__restrict__ as, int M, int nG, float *__restrict__ dst) {
    const size_t total = static_cast<size_t>(M) * nG;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int m = static_cast<int>(i % M);
        const int g = static_cast<int>(i / M);
        dst[i] = as[static_cast<size_t>(m) * nG + g];
    }
}

int grid_for(size_t total, int threads) {
    size_t b = (total + threads - 1) / threads;
    if (b > 148 * 16) b = 148 * 16;
    return b < 1 ? 1 : static_cast<int>(b);
}

int status(cudaError_t e) { return e == cudaSuccess ? 0 : ROCKET_E_DEVICE; }

}  // namespace

extern "C" {

size_t rkb_wpack_codes_bytes(int N, int K, int bits) {
    return rkb::wl_bytes(N, K, 64 * bits / 8);
}

size_t rkb_wpack_scales_bytes(int N, int K) {
    return rkb::wl_bytes(N, K, 2 * sizeof(__half));
}

int rkb_wpack_codes(const int8_t *src, int N, int K, int bits, void *dst, cudaStream_t s) {
    const int nkb = (K + 127) / 128 * 2;
    const size_t total = rkb_wpack_codes_bytes(N, K, bits);
    if (bits == 8)
        pack_codes_i8<<<grid_for(total, 256), 256, 0, s>>>(src, N, K, nkb, static_cast<uint8_t *>(dst), total);
    else if (bits == 4)
        pack_codes_i4<<<grid_for(total, 256), 256, 0, s>>>(src, N, K, nkb, static_cast<uint8_t *>(dst), total);
    else
        return ROCKET_E_UNSUPPORTED;
    return status(cudaGetLastError());
}

int rkb_wpack_scales(const float *b_scale, int N, int K, int group, void *dst, cudaStream_t s) {
    const int nkb = (K + 127) / 128 * 2;
    const int ntiles = rkb::wl_ntiles(N);
    if (ntiles > 65535) return ROCKET_E_SHAPE;
    pack_scales<<<dim3((nkb + 15) / 16, ntiles), rkb::WL_TILE, 0, s>>>(b_scale, N, K, group, nkb,
                                                                 static_cast<uint32_t *>(dst));
    return status(cudaGetLastError());
}

int rkb_wpack_unit_scales(int N, int K, void *dst, cudaStream_t s) {
    return rkb_wpack_scales(nullptr, N, K, 32, dst, s);
}

int rkb_prescale_a(const int8_t *A, const float *a_scale, int M, int K, int group, void *dst,
                   cudaStream_t s) {
    if (K % 16 || M <= 0) return ROCKET_E_SHAPE;
    const int gx = (K / 16 + 255) / 256;
    const int gy = M < 65535 ? M : 65535;
    if (((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0)
        prescale_a<true><<<dim3(gx, gy), 256, 0, s>>>(A, a_scale, M, K, group, static_cast<__half *>(dst));
    else if ((reinterpret_cast<uintptr_t>(dst) & 3) == 0)
        prescale_a<false><<<dim3(gx, gy), 256, 0, s>>>(A, a_scale, M, K, group, static_cast<__half *>(dst));
    else
        return ROCKET_E_SHAPE;
    return status(cudaGetLastError());
}

int rkb_scale_transpose(const float *a_scale, int M, int nG, float *dst, cudaStream_t s) {
    const size_t total = static_cast<size_t>(M) * nG;
    scale_transpose<<<grid_for(total, 256), 256, 0, s>>>(a_scale, M, nG, dst);
    return status(cudaGetLastError());
}

int rkb_gather_row_scale(const float *a_scale, int M, int nG, float *dst, cudaStream_t s) {
    gather_row_scale<<<(M + 255) / 256, 256, 0, s>>>(a_scale, M, nG, dst);
    return status(cudaGetLastError());
}

int rkb_device_sm_count(int dev) {
    static int cache[64];
    if (dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // extern "C"

// ---- dtype helpers for the bf16 / int16 matmul entries -----------------------
namespace {

// fp32 -> bf16 by truncation of the low 16 bits (the reference's bf16 pack
// drops them, include/rocket_matmul.h:510-513)
__global__ void f32_to_bf16_trunc(const uint32_t *__restrict__ src, size_t n, uint16_t *__restrict__ dst) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        dst[i] = static_cast<uint16_t>(src[i] >> 16);
}

// int16 -> (hi, lo) signed bytes with v = 256*hi + lo, v clamped to [-32768, 32639]
// (the reference's exact int16 route, include/rocket_matmul.h:489-499)
__global__ void int16_split(const int16_t *__restrict__ src, size_t n, int8_t *__restrict__ hi,
                            int8_t *__restrict__ lo) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        int v = src[i];
        if (v > 32639) v = 32639;
        const int h = (v + 128) >> 8;          // arithmetic shift = floor division
        hi[i] = static_cast<int8_t>(h);
        lo[i] = static_cast<int8_t>(v - 256 * h);
    }
}

// C = 65536*hh + 256*(hl + lh) + ll in int64
__global__ void int16_combine(const int32_t *__restrict__ hh, const int32_t *__restrict__ hl,
                              const int32_t *__restrict__ lh, const int32_t *__restrict__ ll, size_t n,
                              int64_t *__restrict__ out) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = 65536ll * hh[i] + 256ll * (static_cast<int64_t>(hl[i]) + lh[i]) + ll[i];
}

}  // namespace

extern "C" int rkb_f32_to_bf16(const void *src, size_t n, void *dst, cudaStream_t s) {
    f32_to_bf16_trunc<<<grid_for(n, 256), 256, 0, s>>>(static_cast<const uint32_t *>(src), n,
                                                       static_cast<uint16_t *>(dst));
    return status(cudaGetLastError());
}

extern "C" int rkb_int16_split(const int16_t *src, size_t n, int8_t *hi, int8_t *lo, cudaStream_t s) {
    int16_split<<<grid_for(n, 256), 256, 0, s>>>(src, n, hi, lo);
    return status(cudaGetLastError());
}

extern "C" int rkb_int16_combine(const int32_t *hh, const int32_t *hl, const int32_t *lh, const int32_t *ll,
                                 size_t n, int64_t *out, cudaStream_t s) {
    int16_combine<<<grid_for(n, 256), 256, 0, s>>>(hh, hl, lh, ll, n, out);
    return status(cudaGetLastError());
}

// ---- concatenation of three device arrays (the encoder's fused q/k/v weights) ----
namespace {
__global__ void concat3(const uint4 *__restrict__ a, const uint4 *__restrict__ b, const uint4 *__restrict__ c,
                        size_t n16, uint4 *__restrict__ dst) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < 3 * n16;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t part = i / n16, j = i - part * n16;
        const uint4 *src = part == 0 ? a : part == 1 ? b : c;
        dst[i] = src ? src[j] : make_uint4(0, 0, 0, 0);
    }
}
}  // namespace

// dst = [a | b | c], each `bytes` long (a multiple of 16, all pointers 16-byte
// aligned device memory); a NULL source part is zero-filled.
extern "C" int rkb_concat3(const void *a, const void *b, const void *c, size_t bytes, void *dst, cudaStream_t s) {
    if (bytes % 16 || ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                        reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(dst)) & 15))
        return ROCKET_E_SHAPE;
    const size_t n16 = bytes / 16;
    size_t blocks = (3 * n16 + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    concat3<<<static_cast<int>(blocks), 256, 0, s>>>(static_cast<const uint4 *>(a), static_cast<const uint4 *>(b),
                                                      static_cast<const uint4 *>(c), n16, static_cast<uint4 *>(dst));
    return cudaGetLastError() == cudaSuccess ? 0 : ROCKET_E_DEVICE;
}
