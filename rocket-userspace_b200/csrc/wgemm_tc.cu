// wgemm_tc.cu -- GEMM against resident quantised weights, dequantised in
// registers between the load and the MMA.
//
// Replaces the reference's group-wise and int4 paths (src/rocket_matmul.c
// :2716-2871, :3132-3282; src/rocket_prepacked_int8.c:496-655;
// src/rocket_prepacked_int4.c:490-686), which run one NPU tile per K-group and
// apply a_scale[m,g] * b_scale[n,g] to each int32 partial on the host.
//
// Two modes:
//   MODE_F16  weights (int8 or int4 codes) x fp16 group scales -> fp16 in
//             shared memory, A fp16, tcgen05 kind::f16, fp32 accumulate.  The
//             epilogue applies an optional per-row activation scale.  This is
//             the W4A8 / W8A8 group-wise path.
//   MODE_I8   int4 codes -> int8 in shared memory, A int8, tcgen05 kind::i8,
//             exact int32 accumulate.  This is the raw int4 (W4A4) path.
//
// Roles (448 threads, one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0       producer: TMA for the A tile, bulk copies for the code block
//                and its scale block (both contiguous in the resident layout)
//   warp 1       MMA issuer (single thread), double-buffered TMEM accumulator
//   warps 2..5   epilogue (TMEM -> registers -> global)
//   warps 6..13  dequantisers: raw stage -> 128-byte-swizzled operand tile
//
// Resident weight layout (written by rkb_wpack_codes / rkb_wpack_scales, see
// rkb_wlayout.cuh): for N tile nt (256 rows; the last tile only its own rows)
// and K block kb (64 codes) a contiguous block of rows x 64 codes, row-major; int8 codes are stored offset by
// +128 (u8 = v ^ 0x80) and int4 codes offset by +8 (two per byte, even k in the
// low nibble), so the dequantiser can build fp16 values with byte permutes.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>
#include <cmath>
#include <cstdlib>

#include "rkb_ptx.cuh"
#include "rkb_tmap.h"
#include "rkb_wlayout.cuh"
#include "../src/rkb_kernels.h"
#include "../../include/rocket_npu.h"

namespace rkb {
namespace wq {

constexpr int BM = 128, BN = 256;
constexpr int NUM_THREADS = 448;
constexpr int DEQ_WARP0 = 6, DEQ_WARPS = 8, DEQ_THREADS = DEQ_WARPS * 32;
constexpr int MODE_F16 = 0, MODE_I8 = 1;

template <int MODE, int WBITS>
struct Cfg {
    // raw ring: A tile + code block(s) + scale block, loaded DEPTH stages ahead;
    // dequantised ring: two 256 x 128-byte swizzled B tiles.
    static constexpr int A_BYTES = BM * 128;
    static constexpr int D_BYTES = BN * 128;
    static constexpr int CODE_BLOCK = BN * 64 * WBITS / 8;                 // one 64-wide K block
    static constexpr int CODE_BYTES = (MODE == MODE_F16) ? CODE_BLOCK : 2 * CODE_BLOCK;
    static constexpr int SCALE_BYTES = (MODE == MODE_F16) ? BN * 2 * 2 : 0;
    static constexpr int RAW_BYTES = (A_BYTES + CODE_BYTES + SCALE_BYTES + 1023) / 1024 * 1024;
    static constexpr int TX_BYTES = A_BYTES + CODE_BYTES + SCALE_BYTES;
    static constexpr int DSTAGES = 2;
    static constexpr int BUDGET = 226 * 1024;
    static constexpr int RSTAGES_FIT = (BUDGET - DSTAGES * D_BYTES - 1024 - 512) / RAW_BYTES;
    static constexpr int RSTAGES = RSTAGES_FIT > 6 ? 6 : RSTAGES_FIT;
    static constexpr int NBARS = 2 * RSTAGES + 2 * DSTAGES + 5;
    static constexpr int SMEM = RSTAGES * RAW_BYTES + DSTAGES * D_BYTES + NBARS * 8 + 16 + 1024;
    static_assert(RSTAGES >= 3, "raw ring too shallow");
    static_assert(SMEM <= 232448, "shared memory budget");
};

struct Args {
    int M, N, K;
    int m_tiles, n_tiles, k_blocks;   // k_blocks in units of the MMA K-block
    int kb64_total;                   // 64-wide K blocks per N tile in the layout
    const uint8_t *codes;
    const __half *scales;
    void *C;
    long ldc;
    int out_kind;
    const float *row_scale;
    int *err;
};

RKB_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
RKB_DEV uint32_t lop_and_or(uint32_t a, uint32_t b, uint32_t c) {  // (a & b) | c
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
RKB_DEV uint32_t h2_sub_mul(uint32_t x, uint32_t bias, uint32_t s2) {  // (x - bias) * s2
    __half2 hx = *reinterpret_cast<__half2 *>(&x);
    __half2 hb = *reinterpret_cast<__half2 *>(&bias);
    __half2 hs = *reinterpret_cast<__half2 *>(&s2);
    __half2 r = __hmul2(__hsub2(hx, hb), hs);
    return *reinterpret_cast<uint32_t *>(&r);
}

// 8 int4 codes (one 32-bit word, offset-binary nibbles) -> 8 fp16 (v * s).
RKB_DEV uint4 deq8_i4_f16(uint32_t u, uint32_t s2) {
    const uint32_t e = u & 0x0F0F0F0Fu;          // codes 0,2,4,6
    const uint32_t o = (u >> 4) & 0x0F0F0F0Fu;   // codes 1,3,5,7
    const uint32_t bias = 0x64086408u;           // fp16 1032 = 1024 + 8
    uint4 r;
    r.x = h2_sub_mul(lop_and_or(prmt(e, o, 0x4400u), 0x00FF00FFu, 0x64006400u), bias, s2);
    r.y = h2_sub_mul(lop_and_or(prmt(e, o, 0x5511u), 0x00FF00FFu, 0x64006400u), bias, s2);
    r.z = h2_sub_mul(lop_and_or(prmt(e, o, 0x6622u), 0x00FF00FFu, 0x64006400u), bias, s2);
    r.w = h2_sub_mul(lop_and_or(prmt(e, o, 0x7733u), 0x00FF00FFu, 0x64006400u), bias, s2);
    return r;
}
// 8 int8 codes (two words, offset-binary bytes) -> 8 fp16 (v * s).
RKB_DEV uint4 deq8_i8_f16(uint32_t w0, uint32_t w1, uint32_t s2) {
    const uint32_t k64 = 0x64646464u;
    const uint32_t bias = 0x64806480u;           // fp16 1152 = 1024 + 128
    uint4 r;
    r.x = h2_sub_mul(prmt(w0, k64, 0x5140u), bias, s2);
    r.y = h2_sub_mul(prmt(w0, k64, 0x7362u), bias, s2);
    r.z = h2_sub_mul(prmt(w1, k64, 0x5140u), bias, s2);
    r.w = h2_sub_mul(prmt(w1, k64, 0x7362u), bias, s2);
    return r;
}
// 8 int4 codes (offset-binary nibbles) -> 8 int8 bytes (two words).
RKB_DEV uint2 deq8_i4_i8(uint32_t u) {
    const uint32_t n = u ^ 0x88888888u;                      // two's complement nibbles
    uint32_t e = n & 0x0F0F0F0Fu;
    uint32_t o = (n >> 4) & 0x0F0F0F0Fu;
    e |= (e & 0x08080808u) * 0x1Eu;                          // sign-extend each byte
    o |= (o & 0x08080808u) * 0x1Eu;
    return make_uint2(prmt(e, o, 0x5140u), prmt(e, o, 0x7362u));
}

template <int OUT>
RKB_DEV void store_chunk(const Args &g, int row, int col, const uint32_t (&r)[32]) {
    if (row >= g.M) return;
    if (OUT == RKB_OUT_I32) {
        int32_t *c = static_cast<int32_t *>(g.C) + static_cast<long>(row) * g.ldc + col;
#pragma unroll
        for (int v = 0; v < 4; ++v)
            if (col + 8 * v + 8 <= g.N) {
                int4 *dst = reinterpret_cast<int4 *>(c + 8 * v);
                dst[0] = make_int4(r[8 * v + 0], r[8 * v + 1], r[8 * v + 2], r[8 * v + 3]);
                dst[1] = make_int4(r[8 * v + 4], r[8 * v + 5], r[8 * v + 6], r[8 * v + 7]);
            }
        return;
    }
    const float rs = g.row_scale ? g.row_scale[row] : 1.0f;
    if (OUT == RKB_OUT_F32) {
        float *c = static_cast<float *>(g.C) + static_cast<long>(row) * g.ldc + col;
#pragma unroll
        for (int v = 0; v < 4; ++v)
            if (col + 8 * v + 8 <= g.N) {
                float4 *dst = reinterpret_cast<float4 *>(c + 8 * v);
                dst[0] = make_float4(__uint_as_float(r[8 * v + 0]) * rs, __uint_as_float(r[8 * v + 1]) * rs,
                                     __uint_as_float(r[8 * v + 2]) * rs, __uint_as_float(r[8 * v + 3]) * rs);
                dst[1] = make_float4(__uint_as_float(r[8 * v + 4]) * rs, __uint_as_float(r[8 * v + 5]) * rs,
                                     __uint_as_float(r[8 * v + 6]) * rs, __uint_as_float(r[8 * v + 7]) * rs);
            }
    } else {
        __half *c = static_cast<__half *>(g.C) + static_cast<long>(row) * g.ldc + col;
#pragma unroll
        for (int v = 0; v < 4; ++v)
            if (col + 8 * v + 8 <= g.N) {
                uint32_t h[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __half2 p = __floats2half2_rn(__uint_as_float(r[8 * v + 2 * j]) * rs,
                                                  __uint_as_float(r[8 * v + 2 * j + 1]) * rs);
                    h[j] = *reinterpret_cast<uint32_t *>(&p);
                }
                *reinterpret_cast<uint4 *>(c + 8 * v) = make_uint4(h[0], h[1], h[2], h[3]);
            }
    }
}

template <int MODE, int WBITS, int OUT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
wgemm_kernel(const __grid_constant__ CUtensorMap tmA, const Args g) {
    using C = Cfg<MODE, WBITS>;
    constexpr int RS = C::RSTAGES, DS = C::DSTAGES;
    constexpr uint32_t IDESC = (MODE == MODE_F16) ? idesc_f16_f32acc(BM, BN) : idesc_s8_s32acc(BM, BN);
    constexpr int A_BK_ELEMS = (MODE == MODE_F16) ? 64 : 128;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    // layout: [DS dequantised B tiles][RS raw stages][barriers]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + DS * C::D_BYTES + RS * C::RAW_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBARS);
    const uint32_t sbase = smem_u32(smem);
    auto sD = [&](int d) { return sbase + d * C::D_BYTES; };
    auto pD = [&](int d) { return smem + d * C::D_BYTES; };
    auto rbase = [&](int r) { return DS * C::D_BYTES + r * C::RAW_BYTES; };
    auto sA = [&](int r) { return sbase + rbase(r); };
    auto sCode = [&](int r) { return sbase + rbase(r) + C::A_BYTES; };
    auto sScale = [&](int r) { return sbase + rbase(r) + C::A_BYTES + C::CODE_BYTES; };
    auto pCode = [&](int r) { return smem + rbase(r) + C::A_BYTES; };
    auto pScale = [&](int r) {
        return reinterpret_cast<const uint16_t *>(smem + rbase(r) + C::A_BYTES + C::CODE_BYTES);
    };
    auto raw_full = [&](int r) { return smem_u32(&bars[r]); };
    auto raw_empty = [&](int r) { return smem_u32(&bars[RS + r]); };
    auto deq_full = [&](int d) { return smem_u32(&bars[2 * RS + d]); };
    auto deq_empty = [&](int d) { return smem_u32(&bars[2 * RS + DS + d]); };
    auto tfull_bar = [&](int b) { return smem_u32(&bars[2 * RS + 2 * DS + b]); };
    auto tempty_bar = [&](int b) { return smem_u32(&bars[2 * RS + 2 * DS + 2 + b]); };
    const uint32_t drain_bar = smem_u32(&bars[2 * RS + 2 * DS + 4]);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmA);
        for (int r = 0; r < RS; ++r) {
            mbar_init(raw_full(r), 1);
            mbar_init(raw_empty(r), 1);
        }
        for (int d = 0; d < DS; ++d) {
            mbar_init(deq_full(d), DEQ_WARPS);
            mbar_init(deq_empty(d), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 128);
        }
        mbar_init(drain_bar, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_tiles = g.m_tiles * g.n_tiles;

    if (warp == 0) {
        if (lane == 0) {
            int r = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int mt = t % g.m_tiles, nt = t / g.m_tiles;
                // ragged layout: the last N tile stores only its own rows (the
                // rest of the stage keeps stale, finite data; those rows are
                // never stored)
                constexpr int RB = 64 * WBITS / 8;
                const int rows = wl_rows(g.N, nt);
                const uint32_t blk = static_cast<uint32_t>(rows * RB);
                const uint32_t tx = C::A_BYTES + (MODE == MODE_F16 ? blk + rows * 4 : 2 * blk);
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    if (!mbar_wait(raw_empty(r), ph ^ 1, g.err, ERR_WAIT_PRODUCER)) { ok = false; break; }
                    mbar_arrive_expect_tx(raw_full(r), tx);
                    tma_load_2d(sA(r), &tmA, kb * A_BK_ELEMS, mt * BM, raw_full(r));
                    if (MODE == MODE_F16) {
                        bulk_load(sCode(r), g.codes + wl_block(g.N, g.kb64_total, nt, kb, RB), blk, raw_full(r));
                        bulk_load(sScale(r),
                                  reinterpret_cast<const uint8_t *>(g.scales) + wl_block(g.N, g.kb64_total, nt, kb, 4),
                                  rows * 4, raw_full(r));
                    } else {
                        // two 64-wide K blocks per 128-wide MMA K block, 256 rows apart in shared memory
                        bulk_load(sCode(r), g.codes + wl_block(g.N, g.kb64_total, nt, 2 * kb, RB), blk, raw_full(r));
                        bulk_load(sCode(r) + Cfg<MODE_F16, WBITS>::CODE_BLOCK,
                                  g.codes + wl_block(g.N, g.kb64_total, nt, 2 * kb + 1, RB), blk, raw_full(r));
                    }
                    if (++r == RS) { r = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int r = 0, d = 0;
            uint32_t rph = 0, dph = 0;
            bool ok = true;
            int it = 0;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
                const int b = it & 1;
                const uint32_t aph = (it >> 1) & 1;
                if (!mbar_wait(tempty_bar(b), aph ^ 1, g.err, ERR_WAIT_MMA_ACC)) { ok = false; break; }
                tc_fence_after();
                const uint32_t dcol = tmem_base + b * BN;
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    // deq_full(d) completes only after the dequantisers saw raw_full(r),
                    // so the A tile of raw stage r has landed as well
                    if (!mbar_wait(deq_full(d), dph, g.err, ERR_WAIT_MMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128(sA(r));
                    const uint64_t bdesc = smem_desc_sw128(sD(d));
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t koff = static_cast<uint64_t>((k * 32) >> 4);
                        const uint32_t acc = (kb | k) != 0;
                        if (MODE == MODE_F16) tc_mma_f16(dcol, adesc + koff, bdesc + koff, IDESC, acc);
                        else                  tc_mma_i8(dcol, adesc + koff, bdesc + koff, IDESC, acc);
                    }
                    tc_commit(raw_empty(r));
                    tc_commit(deq_empty(d));
                    if (++r == RS) { r = 0; rph ^= 1; }
                    if (++d == DS) { d = 0; dph ^= 1; }
                }
                if (ok) tc_commit(tfull_bar(b));
            }
            (void)rph;
            if (!ok) {
                tc_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0);
            }
        }
    } else if (warp < DEQ_WARP0) {
        const int q = warp & 3;
        int it = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
            const int b = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!mbar_wait_warp(tfull_bar(b), aph, g.err, ERR_WAIT_EPILOGUE)) break;
            tc_fence_after();
            const int mt = t % g.m_tiles, nt = t / g.m_tiles;
            const int row = mt * BM + q * 32 + lane;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * BN;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t rr[32];
                tmem_ld32(tbase + c, rr);
                tmem_ld_wait();
                const int col = nt * BN + c;
                if (col < g.N) store_chunk<OUT>(g, row, col, rr);
            }
            tc_fence_before();
            mbar_arrive(tempty_bar(b));
        }
    } else {
        // Dequantisers: 256 threads turn raw stage r into dequantised tile d.
        // Chunk id = i * 256 + tid covers (row, 16-byte chunk c); the swizzled
        // destination is row * 128 + ((c ^ (row & 7)) << 4).
        const int tid = threadIdx.x - DEQ_WARP0 * 32;
        int r = 0, d = 0;
        uint32_t rph = 0, dph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < g.k_blocks; ++kb) {
                if (!mbar_wait_warp(raw_full(r), rph, g.err, ERR_WAIT_DEQUANT) ||
                    !mbar_wait_warp(deq_empty(d), dph ^ 1, g.err, ERR_WAIT_DEQUANT)) { ok = false; break; }
                const uint8_t *code = pCode(r);
                uint8_t *dst = pD(d);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int id = i * DEQ_THREADS + tid;
                    const int row = id >> 3, c = id & 7;
                    uint4 out;
                    if (MODE == MODE_F16) {
                        const uint16_t sh = pScale(r)[row * 2 + (c >> 2)];
                        const uint32_t s2 = static_cast<uint32_t>(sh) | (static_cast<uint32_t>(sh) << 16);
                        if (WBITS == 4) {
                            const uint32_t u = *reinterpret_cast<const uint32_t *>(code + row * 32 + c * 4);
                            out = deq8_i4_f16(u, s2);
                        } else {
                            const uint2 w = *reinterpret_cast<const uint2 *>(code + row * 64 + c * 8);
                            out = deq8_i8_f16(w.x, w.y, s2);
                        }
                    } else {
                        // 16 int4 codes k = 16c .. 16c+15: block (c >> 2), bytes (c & 3) * 8
                        const uint2 w = *reinterpret_cast<const uint2 *>(
                            code + (c >> 2) * Cfg<MODE_F16, 4>::CODE_BLOCK + row * 32 + (c & 3) * 8);
                        const uint2 lo = deq8_i4_i8(w.x), hi = deq8_i4_i8(w.y);
                        out = make_uint4(lo.x, lo.y, hi.x, hi.y);
                    }
                    *reinterpret_cast<uint4 *>(dst + row * 128 + ((c ^ (row & 7)) << 4)) = out;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(deq_full(d));
                if (++r == RS) { r = 0; rph ^= 1; }
                if (++d == DS) { d = 0; dph ^= 1; }
            }
        }
    }

    tc_fence_before();
    __syncwarp();   // reconverge role-divergent lanes: the barrier below is warp-aligned
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * BN);
    }
}

template <int MODE, int WBITS, int OUT>
int launch(const rkb_wgemm_desc *d, int *err, cudaStream_t stream) {
    using C = Cfg<MODE, WBITS>;
    static std::once_flag attr_once[16];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 15], [] {
        cudaFuncSetAttribute(wgemm_kernel<MODE, WBITS, OUT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    CUtensorMap ta;
    if (MODE == MODE_F16) {
        if (make_tmap_2d(&ta, d->A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, d->K, d->M, d->lda, 64, BM))
            return ROCKET_E_SHAPE;
    } else {
        if (make_tmap_2d(&ta, d->A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, d->K, d->M, d->lda, 128, BM))
            return ROCKET_E_SHAPE;
    }
    Args g;
    g.M = d->M; g.N = d->N; g.K = d->K;
    g.m_tiles = (d->M + BM - 1) / BM;
    g.n_tiles = (d->N + BN - 1) / BN;
    const int kp = (d->K + 127) / 128 * 128;   // packed K (multiple of 128)
    g.kb64_total = kp / 64;
    g.k_blocks = (MODE == MODE_F16) ? kp / 64 : kp / 128;
    g.codes = static_cast<const uint8_t *>(d->Wq);
    g.scales = static_cast<const __half *>(d->Ws);
    g.C = d->C; g.ldc = d->ldc; g.out_kind = d->out_kind;
    g.row_scale = d->row_scale;
    g.err = err;
    const int tiles = g.m_tiles * g.n_tiles;
    const int sms = rkb_device_sm_count(dev);
    const int grid = tiles < sms ? tiles : sms;
    wgemm_kernel<MODE, WBITS, OUT><<<grid, NUM_THREADS, C::SMEM, stream>>>(ta, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "rkb wgemm launch: %s\n", cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    return 0;
}


}  // namespace wq
}  // namespace rkb

extern "C" int rkb_wgemm_run(const rkb_wgemm_desc *d, int *err, cudaStream_t stream) {
    using namespace rkb::wq;
    if (d->M <= 0 || d->N <= 0 || d->K <= 0 || (d->N & 7) || (d->ldc & 7)) return ROCKET_E_SHAPE;
#define RKB_WQ(MODE, BITS, OUT) return launch<MODE, BITS, OUT>(d, err, stream)
    if (d->a_f16) {
        static const bool smem_b = getenv("ROCKET_WGEMM_SMEM_B") != nullptr;
        if (!smem_b) return rkb_wgemm_ts_run(d, err, stream);
        if (d->w_bits == 4) {
            if (d->out_kind == RKB_OUT_F32) { RKB_WQ(MODE_F16, 4, RKB_OUT_F32); }
            if (d->out_kind == RKB_OUT_F16) { RKB_WQ(MODE_F16, 4, RKB_OUT_F16); }
        } else if (d->w_bits == 8) {
            if (d->out_kind == RKB_OUT_F32) { RKB_WQ(MODE_F16, 8, RKB_OUT_F32); }
            if (d->out_kind == RKB_OUT_F16) { RKB_WQ(MODE_F16, 8, RKB_OUT_F16); }
        }
    } else if (d->w_bits == 4 && d->out_kind == RKB_OUT_I32) {
        RKB_WQ(MODE_I8, 4, RKB_OUT_I32);
    }
#undef RKB_WQ
    return ROCKET_E_UNSUPPORTED;
}
