// gemm_tc.cu -- dense C[M,N] = A[M,K] * B[N,K]^T on the sm_100a tensor cores.
//
// This is the kernel behind rocket_matmul_fp16 / rocket_matmul_int8 and their
// resident and multi-GPU forms (reference src/rocket_matmul.c:975-1105 and
// :2439-2627 run the same contraction as NPU tile programs with host K-accum).
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128-byte-swizzled A (128 x 128 B) and B (BN x 128 B)
//               K-blocks into a STAGES-deep shared-memory ring.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (kind::f16 with fp32
//               accumulate, or kind::i8 with exact int32 accumulate) into a TMEM
//               accumulator of 128 lanes x BN columns; two accumulators
//               alternate so the epilogue of tile i overlaps the MMAs of i+1.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (warp w owns TMEM
//               lanes 32*(w%4)..+31 = output rows), convert, store to global
//               (directly, or staged in shared memory and written by TMA).
// The CTA-pair kernel (gemm2_kernel, further down) computes 256-row tiles on
// two SMs with tcgen05.mma.cta_group::2 and has 8 epilogue warps; it also
// carries the int8 stream-K tail and the fp16 split-K slabs.
// Both operands are K-major ("TN"), which is the layout the reference API
// defines (B is [N,K] row-major), so no transposes are ever made.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "rkb_ptx.cuh"
#include "rkb_tmap.h"
#include "../src/rkb_kernels.h"
#include "../../include/rocket_npu.h"

namespace rkb {
namespace dense {

// Per input kind: element size, instruction descriptor, TMA element type.
template <int KIND> struct Kind;
template <> struct Kind<RKB_IN_F16> {
    static constexpr int ESIZE = 2;
    static constexpr CUtensorMapDataType DT = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    static constexpr uint32_t idesc(int m, int n) { return idesc_f16_f32acc(m, n); }
};
template <> struct Kind<RKB_IN_BF16> {
    static constexpr int ESIZE = 2;
    static constexpr CUtensorMapDataType DT = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    static constexpr uint32_t idesc(int m, int n) { return idesc_f32acc_fmt(1, m, n); }
};
template <> struct Kind<RKB_IN_TF32> {
    static constexpr int ESIZE = 4;
    static constexpr CUtensorMapDataType DT = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    static constexpr uint32_t idesc(int m, int n) { return idesc_f32acc_fmt(2, m, n); }
};
template <> struct Kind<RKB_IN_I8> {
    static constexpr int ESIZE = 1;
    static constexpr CUtensorMapDataType DT = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    static constexpr uint32_t idesc(int m, int n) { return idesc_s8_s32acc(m, n); }
};

constexpr int BM = 128;            // UMMA M (cta_group::1)
constexpr int BK_BYTES = 128;      // one 128-byte swizzle row per K-block
constexpr int NUM_THREADS = 192;   // 6 warps (single-CTA kernel)
// CTA-pair kernel: producer, MMA and 8 epilogue warps -- two per TMEM lane
// quarter, each draining half of the tile's columns, so epilogue-heavy GEMMs
// (short K with bias / GELU / residual) keep up with the mainloop
constexpr int EPI_WARPS2 = 8;
constexpr int NUM_THREADS2 = (2 + EPI_WARPS2) * 32;
constexpr int PREFETCH = 12;       // default K-blocks of L2 prefetch ahead of the current load

template <int BN>
struct Cfg {
    static constexpr int A_BYTES = BM * BK_BYTES;
    static constexpr int B_BYTES = BN * BK_BYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BN == 256) ? 4 : 6;
    static constexpr int TMEM_COLS = 2 * BN;   // two accumulators
    static constexpr int STG_BYTES = 4 * 2 * 4096;   // epilogue: 4 warps x 2 chunk buffers
    static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
    static constexpr int SMEM = STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES + 1024;
};

struct Args {
    int M, N, K;
    int m_tiles, n_tiles, k_blocks;
    void *C;
    long ldc;
    const float *row_scale;
    const float *col_scale;
    const __half *bias;
    const __half *residual;
    long ldr;
    int act;
    int k_splits, kb_per_split;   // split-K: unit t -> (split, tile); partials at C + split*split_stride
    long split_stride;
    int tma_store;                // C written through the tensor map (staged, full lines)
    int prefetch;                 // K-blocks of L2 prefetch ahead (0 = none)
    // stream-K tail (pair kernel): sk_W full waves of whole tiles, then the
    // K-iterations of the remaining sk_R tiles split evenly, sk_L per pair
    int sk, sk_W, sk_R, sk_L;
    void *sk_part;                // per tail tile a 256 x BN sum buffer (zeroed per launch)
    int *sk_cnt;                  // per tail tile 8 arrival counters (zeroed per launch)
    int *err;
};

RKB_DEV float apply_act(float v, int act) {
    if (act == RKB_ACT_GELU) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    if (act == RKB_ACT_SILU) return v / (1.0f + expf(-v));
    return v;
}

// Output words of 32 consecutive columns of one row with the fused epilogue
// applied: 32 words for 4-byte outputs, 16 (fp16 pairs) for fp16.  Rows past M
// and vectors past N read nothing; their words are never stored.
template <int OUT>
RKB_DEV void pack_chunk(const Args &g, int row, int col, uint32_t (&r)[32]) {
    const bool in = row < g.M;
    if (OUT == RKB_OUT_I32) return;
    const float rs = (in && g.row_scale) ? g.row_scale[row] : 1.0f;
    if (OUT == RKB_OUT_F32) {
        if (!g.row_scale && !g.col_scale) return;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float cs = (g.col_scale && col + j < g.N) ? g.col_scale[col + j] : 1.0f;
            r[j] = __float_as_uint(__uint_as_float(r[j]) * rs * cs);
        }
        return;
    }
    const __half *res = (in && g.residual) ? g.residual + static_cast<long>(row) * g.ldr + col : nullptr;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const bool vin = col + 8 * v + 8 <= g.N;
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float a = __uint_as_float(r[8 * v + j]) * rs;
            if (g.col_scale && vin) a *= g.col_scale[col + 8 * v + j];
            if (g.bias && vin) a += __half2float(g.bias[col + 8 * v + j]);
            f[j] = apply_act(a, g.act);
        }
        if (res && vin) {
            const uint4 rv = *reinterpret_cast<const uint4 *>(res + 8 * v);
            const __half *rh = reinterpret_cast<const __half *>(&rv);
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] += __half2float(rh[j]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 p = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
            r[4 * v + j] = *reinterpret_cast<uint32_t *>(&p);
        }
    }
}

// Stage one packed 32-row x 32-column chunk (this warp's rows) in the swizzled
// layout the C tensor map expects -- 128-byte rows with the 128-byte swizzle for
// 4-byte outputs, 64-byte rows with the 64-byte swizzle for fp16 -- and store it
// with one TMA instruction.  Both patterns keep the one-row-per-thread writes
// free of bank conflicts.
template <int OUT>
RKB_DEV void stage_store(const CUtensorMap *tmC, uint32_t buf, int lane, const uint32_t (&w)[32],
                         int col, int row0, int plane = -1) {
    if (OUT == RKB_OUT_F16) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t a = buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(w[4 * j]), "r"(w[4 * j + 1]),
                         "r"(w[4 * j + 2]), "r"(w[4 * j + 3]) : "memory");
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t a = buf + lane * 128 + ((j ^ (lane & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(w[4 * j]), "r"(w[4 * j + 1]),
                         "r"(w[4 * j + 2]), "r"(w[4 * j + 3]) : "memory");
        }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        if (plane < 0) tma_store_2d(tmC, buf, col, row0);
        else tma_store_3d(tmC, buf, col, row0, plane);   // split-K slab
        bulk_commit();
    }
}

template <int OUT>
RKB_DEV void store_chunk(const Args &g, int row, int col, const uint32_t (&r)[32]) {
    // 32 consecutive columns of one output row; N % 8 == 0 so a vector of 8
    // is either fully inside or fully outside.
    if (row >= g.M) return;
    float rs = g.row_scale ? g.row_scale[row] : 1.0f;
    if (OUT == RKB_OUT_I32) {
        int32_t *c = static_cast<int32_t *>(g.C) + static_cast<long>(row) * g.ldc + col;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            if (col + 8 * v + 8 <= g.N) {
                int4 *dst = reinterpret_cast<int4 *>(c + 8 * v);
                dst[0] = make_int4(r[8 * v + 0], r[8 * v + 1], r[8 * v + 2], r[8 * v + 3]);
                dst[1] = make_int4(r[8 * v + 4], r[8 * v + 5], r[8 * v + 6], r[8 * v + 7]);
            }
        }
    } else if (OUT == RKB_OUT_F32) {
        float *c = static_cast<float *>(g.C) + static_cast<long>(row) * g.ldc + col;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            if (col + 8 * v + 8 <= g.N) {
                float f[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float cs = g.col_scale ? g.col_scale[col + 8 * v + j] : 1.0f;
                    f[j] = __uint_as_float(r[8 * v + j]) * rs * cs;
                }
                float4 *dst = reinterpret_cast<float4 *>(c + 8 * v);
                dst[0] = make_float4(f[0], f[1], f[2], f[3]);
                dst[1] = make_float4(f[4], f[5], f[6], f[7]);
            }
        }
    } else {
        __half *c = static_cast<__half *>(g.C) + static_cast<long>(row) * g.ldc + col;
        const __half *res = g.residual ? g.residual + static_cast<long>(row) * g.ldr + col : nullptr;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            if (col + 8 * v + 8 <= g.N) {
                float f[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float a = __uint_as_float(r[8 * v + j]) * rs;
                    if (g.col_scale) a *= g.col_scale[col + 8 * v + j];
                    if (g.bias) a += __half2float(g.bias[col + 8 * v + j]);
                    f[j] = apply_act(a, g.act);
                }
                if (res) {
                    const uint4 rv = *reinterpret_cast<const uint4 *>(res + 8 * v);
                    const __half *rh = reinterpret_cast<const __half *>(&rv);
#pragma unroll
                    for (int j = 0; j < 8; ++j) f[j] += __half2float(rh[j]);
                }
                uint32_t h[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __half2 p = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
                    h[j] = *reinterpret_cast<uint32_t *>(&p);
                }
                *reinterpret_cast<uint4 *>(c + 8 * v) = make_uint4(h[0], h[1], h[2], h[3]);
            }
        }
    }
}

template <int KIND, int OUT, int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmC, const Args g) {
    using C = Cfg<BN>;
    constexpr int STAGES = C::STAGES;
    constexpr int BK_ELEMS = BK_BYTES / Kind<KIND>::ESIZE;
    constexpr int UMMA_K_BYTES = 32;                      // 16 fp16/bf16, 8 tf32 or 32 int8 per MMA
    constexpr int K_STEPS = BK_BYTES / UMMA_K_BYTES;      // 4 MMAs per K-block
    constexpr uint32_t IDESC = Kind<KIND>::idesc(BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * C::STAGE_BYTES + C::STG_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 5);
    const uint32_t smem_base = smem_u32(smem);
    const uint32_t stg_base = smem_base + STAGES * C::STAGE_BYTES;
    auto sA = [&](int s) { return smem_base + s * C::STAGE_BYTES; };
    auto sB = [&](int s) { return smem_base + s * C::STAGE_BYTES + C::A_BYTES; };
    auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
    auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
    auto tfull_bar = [&](int b) { return smem_u32(&bars[2 * STAGES + b]); };
    auto tempty_bar = [&](int b) { return smem_u32(&bars[2 * STAGES + 2 + b]); };
    const uint32_t drain_bar = smem_u32(&bars[2 * STAGES + 4]);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (g.tma_store) prefetch_tmap(&tmC);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 128);
        }
        mbar_init(drain_bar, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_tiles = g.m_tiles * g.n_tiles;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int mt = t % g.m_tiles, nt = t / g.m_tiles;
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    if (g.prefetch && kb + g.prefetch < g.k_blocks) {   // L2 prefetch beyond the ring
                        tma_prefetch_2d(&tmA, (kb + g.prefetch) * BK_ELEMS, mt * BM);
                        tma_prefetch_2d(&tmB, (kb + g.prefetch) * BK_ELEMS, nt * BN);
                    }
                    if (!mbar_wait(empty_bar(s), ph ^ 1, g.err, ERR_WAIT_PRODUCER)) { ok = false; break; }
                    mbar_arrive_expect_tx(full_bar(s), C::STAGE_BYTES);
                    tma_load_2d(sA(s), &tmA, kb * BK_ELEMS, mt * BM, full_bar(s));
                    tma_load_2d(sB(s), &tmB, kb * BK_ELEMS, nt * BN, full_bar(s));
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int it = 0;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
                const int b = it & 1;
                const uint32_t aph = (it >> 1) & 1;
                if (!mbar_wait(tempty_bar(b), aph ^ 1, g.err, ERR_WAIT_MMA_ACC)) { ok = false; break; }
                tc_fence_after();
                const uint32_t dcol = tmem_base + b * BN;
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    if (!mbar_wait(full_bar(s), ph, g.err, ERR_WAIT_MMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128(sA(s));
                    const uint64_t bdesc = smem_desc_sw128(sB(s));
#pragma unroll
                    for (int k = 0; k < K_STEPS; ++k) {
                        const uint64_t koff = static_cast<uint64_t>((k * UMMA_K_BYTES) >> 4);
                        const uint32_t acc = (kb | k) != 0;
                        if (KIND == RKB_IN_I8)        tc_mma_i8(dcol, adesc + koff, bdesc + koff, IDESC, acc);
                        else if (KIND == RKB_IN_TF32) tc_mma_tf32(dcol, adesc + koff, bdesc + koff, IDESC, acc);
                        else                          tc_mma_f16(dcol, adesc + koff, bdesc + koff, IDESC, acc);
                    }
                    tc_commit(empty_bar(s));
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                if (ok) tc_commit(tfull_bar(b));
            }
            if (!ok) {
                // Error path: let every MMA already issued finish (bounded wait)
                // before the accumulators are freed.
                tc_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0);
            }
        }
    } else {
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        int it = 0;
        uint32_t nstore = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
            const int b = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!mbar_wait_warp(tfull_bar(b), aph, g.err, ERR_WAIT_EPILOGUE)) break;
            tc_fence_after();
            const int mt = t % g.m_tiles, nt = t / g.m_tiles;
            const int row = mt * BM + q * 32 + lane;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * BN;
            if (g.tma_store) {
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c, r);
                    tmem_ld_wait();
                    if (c + 32 == BN) {   // accumulator drained: release it before the last store
                        tc_fence_before();
                        mbar_arrive(tempty_bar(b));
                    }
                    const int col = nt * BN + c;
                    if (col >= g.N) continue;
                    pack_chunk<OUT>(g, row, col, r);
                    // fp16 chunks are 2 KB: four buffers in the warp's 8 KB, else two
                    constexpr int NBUF = OUT == RKB_OUT_F16 ? 4 : 2;
                    const uint32_t buf = stg_base + q * 8192 + (nstore % NBUF) * (8192 / NBUF);
                    if (lane == 0) bulk_wait_read<NBUF - 1>();   // the store that used buf has read it
                    __syncwarp();
                    stage_store<OUT>(&tmC, buf, lane, r, col, row - lane);
                    ++nstore;
                }
                continue;
            }
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t r[32];
                tmem_ld32(tbase + c, r);
                tmem_ld_wait();
                const int col = nt * BN + c;
                if (col < g.N) store_chunk<OUT>(g, row, col, r);
            }
            tc_fence_before();
            mbar_arrive(tempty_bar(b));
        }
        if (lane == 0 && g.tma_store) bulk_wait<0>();
    }

    tc_fence_before();
    __syncwarp();   // reconverge role-divergent lanes: the barrier below is warp-aligned
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// Stream-K tail plan for the pair kernel: when whole tiles leave the last
// wave under 90% full, the K-iterations of the tail tiles are spread over all
// pairs.  ROCKET_GEMM_STREAMK=0 turns it off.
struct SkPlan {
    int on, P, W, R, L;
    size_t part_bytes, cnt_bytes;
};
inline SkPlan sk_plan(int M, int N, int K, int esize, int BN, int sms) {
    static const int env = getenv("ROCKET_GEMM_STREAMK") ? atoi(getenv("ROCKET_GEMM_STREAMK")) : 1;
    SkPlan p{};
    const int P = sms / 2;
    // int8 only: its int32 sums are exact in any order; float sums would depend
    // on the order the segments arrive in
    if (!env || esize != 1 || P < 1) return p;
    const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN);
    const int kb = (K * esize + BK_BYTES - 1) / BK_BYTES;
    if (tiles % P == 0) return p;
    const int waves = (tiles + P - 1) / P;
    if (tiles >= 0.9 * waves * P) return p;
    p.P = P;
    p.W = tiles / P;
    p.R = tiles - p.W * P;
    p.L = (p.R * kb + P - 1) / P;
    if (p.L < 4) return SkPlan{};
    p.on = 1;
    p.part_bytes = static_cast<size_t>(p.R) * 2 * BM * BN * 4;
    p.cnt_bytes = (static_cast<size_t>(p.R) * 2 * EPI_WARPS2 * 4 + 255) & ~static_cast<size_t>(255);
    return p;
}

// L2 prefetch distance in K-blocks (ROCKET_GEMM_PREFETCH, default PREFETCH)
inline int prefetch_distance() {
    static const int v = getenv("ROCKET_GEMM_PREFETCH") ? atoi(getenv("ROCKET_GEMM_PREFETCH")) : PREFETCH;
    return v < 0 ? 0 : v;
}

// Tensor map for the staged TMA-store epilogue: 32 x 32 boxes, 128-byte swizzle
// for 4-byte outputs, 64-byte for fp16.  Returns 1 when C is written that way:
// 16-byte aligned base and row pitch, and at least 16 K-blocks per tile -- with
// shorter K the epilogue is on the critical path and the staged stores (whose
// shared-memory reads queue behind the producer's next-tile loads on the same
// TMA unit) measured slower than direct stores; so did fused bias / residual /
// activation epilogues at every K tried.  ROCKET_GEMM_DIRECT_STORE=1 forces
// direct stores, =0 staged stores whenever the layout allows.
template <int OUT>
int c_store_map(CUtensorMap *tc, int M, int N, void *C, long ldc, int k_blocks, bool fused) {
    static const int env = getenv("ROCKET_GEMM_DIRECT_STORE") ? atoi(getenv("ROCKET_GEMM_DIRECT_STORE")) : -1;
    memset(tc, 0, sizeof *tc);
    const int osize = OUT == RKB_OUT_F16 ? 2 : 4;
    if (env == 1 || (env < 0 && (k_blocks < 16 || fused))) return 0;
    if ((reinterpret_cast<uintptr_t>(C) & 15) || ((ldc * osize) & 15)) return 0;
    const CUtensorMapDataType odt = OUT == RKB_OUT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                  : OUT == RKB_OUT_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                       : CU_TENSOR_MAP_DATA_TYPE_INT32;
    const CUtensorMapSwizzle sw = OUT == RKB_OUT_F16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    return make_tmap_2d(tc, C, odt, osize, N, M, ldc, 32, 32, sw) == 0 ? 1 : 0;
}

template <int KIND, int OUT, int BN>
int launch(const rkb_gemm_desc *d, int *err, cudaStream_t stream) {
    using C = Cfg<BN>;
    static std::once_flag attr_once[16];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 15], [] {
        cudaFuncSetAttribute(gemm_kernel<KIND, OUT, BN>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    const int esize = Kind<KIND>::ESIZE;
    const CUtensorMapDataType dt = Kind<KIND>::DT;
    CUtensorMap ta, tb;
    if (make_tmap_2d(&ta, d->A, dt, esize, d->K, d->M, d->lda, BK_BYTES / esize, BM) ||
        make_tmap_2d(&tb, d->B, dt, esize, d->K, d->N, d->ldb, BK_BYTES / esize, BN))
        return ROCKET_E_SHAPE;
    Args g;
    g.M = d->M; g.N = d->N; g.K = d->K;
    g.m_tiles = (d->M + BM - 1) / BM;
    g.n_tiles = (d->N + BN - 1) / BN;
    g.k_blocks = (d->K * esize + BK_BYTES - 1) / BK_BYTES;
    g.C = d->C; g.ldc = d->ldc;
    g.row_scale = d->row_scale; g.col_scale = d->col_scale;
    g.bias = static_cast<const __half *>(d->bias);
    g.residual = static_cast<const __half *>(d->residual);
    g.ldr = d->ldr; g.act = d->act;
    g.k_splits = 1; g.kb_per_split = g.k_blocks; g.split_stride = 0;
    g.err = err;
    CUtensorMap tc;
    g.tma_store = c_store_map<OUT>(&tc, d->M, d->N, g.C, g.ldc, g.k_blocks,
                                  g.bias || g.residual || g.act != RKB_ACT_NONE);
    g.prefetch = prefetch_distance();
    const int tiles = g.m_tiles * g.n_tiles;
    const int sms = rkb_device_sm_count(dev);
    const int grid = tiles < sms ? tiles : sms;
    gemm_kernel<KIND, OUT, BN><<<grid, NUM_THREADS, C::SMEM, stream>>>(ta, tb, tc, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "rkb gemm launch: %s\n", cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    return 0;
}


// Work units of one CTA pair: (tile, K-block range).  Without stream-K: tiles
// pair, pair + P, ... (with the opt-in split-K ranges).  With stream-K: sk_W
// whole tiles per pair, then this pair's contiguous share of the tail's
// flattened (tile, K-block) iterations, cut at tile boundaries.  A cut tile
// ("split" unit) is finished by whichever of its segments arrives last.
// Stream-K sum buffers: per tail tile 256 rows x BN words, word-interleaved so
// that warp w of CTA r adds and reads its 32 rows x 32-column chunk c with
// coalesced 128-byte lines: word ((((r * 4 + w) * (BN / 32) + c) * 32 + j) * 32 + lane).
struct Unit {
    int tile, k0, k1;
    int split, tl;            // stream-K: split segment, tail tile index (split-K: slab index)
};
struct UnitIter {
    int pair, P, i, it, end;
};
RKB_DEV void units_begin(const Args &g, int pair, int P, UnitIter &u) {
    u.pair = pair; u.P = P; u.i = 0;
    u.it = pair * g.sk_L;
    const int tot = g.sk_R * g.k_blocks;
    u.end = u.it + g.sk_L < tot ? u.it + g.sk_L : tot;
}
RKB_DEV bool units_next(const Args &g, int mn_tiles, UnitIter &s, Unit &u) {
    u.split = 0; u.tl = 0;
    if (!g.sk) {
        const int t = s.pair + s.i * s.P;
        if (t >= mn_tiles * g.k_splits) return false;
        ++s.i;
        u.tile = t % mn_tiles;
        u.k0 = (t / mn_tiles) * g.kb_per_split;
        const int e = u.k0 + g.kb_per_split;
        u.k1 = e < g.k_blocks ? e : g.k_blocks;
        u.tl = t / mn_tiles;   // split-K slab index
        return true;
    }
    if (s.i < g.sk_W) {
        u.tile = s.pair + s.i * s.P;
        ++s.i;
        u.k0 = 0; u.k1 = g.k_blocks;
        return true;
    }
    if (s.it >= s.end) return false;
    const int kb = g.k_blocks;
    const int tau = s.it / kb, k0 = s.it % kb;
    const int k1 = k0 + (s.end - s.it) < kb ? k0 + (s.end - s.it) : kb;
    u.tile = g.sk_W * s.P + tau;
    u.k0 = k0; u.k1 = k1;
    u.split = !(k0 == 0 && k1 == kb);
    u.tl = tau;
    s.it += k1 - k0;
    return true;
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs (two SMs) computes a 256 x BN tile
// with tcgen05.mma.cta_group::2 (M = 256).  CTA r loads rows r*128..+127 of the
// A tile and rows r*BN/2..+BN/2-1 of the B tile into its own shared memory;
// the leader's MMA reads both halves, and each CTA's TMEM receives its 128
// output rows x BN columns.  Per SM this moves 16 + BN/2*128/1024 KB per
// K-block instead of 16 + BN*128/1024 KB, which is what the single-CTA kernel
// is limited by (L2 -> SM operand bandwidth).
template <int BN>
struct Cfg2 {
    static constexpr int BNH = BN / 2;
    static constexpr int A_BYTES = BM * BK_BYTES;
    static constexpr int B_BYTES = BNH * BK_BYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BN == 256) ? 6 : 8;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int STG_BYTES = 4 * 2 * 4096;   // epilogue: 4 warps x 2 chunk buffers
    static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
    static constexpr int SMEM = STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES + 1024;
};

template <int KIND, int OUT, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS2, 1)
gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
             const __grid_constant__ CUtensorMap tmC, const Args g) {
    using C = Cfg2<BN>;
    constexpr int STAGES = C::STAGES;
    constexpr int BK_ELEMS = BK_BYTES / Kind<KIND>::ESIZE;
    constexpr uint32_t IDESC = Kind<KIND>::idesc(2 * BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * C::STAGE_BYTES + C::STG_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 5);
    const uint32_t smem_base = smem_u32(smem);
    const uint32_t stg_base = smem_base + STAGES * C::STAGE_BYTES;
    auto sA = [&](int s) { return smem_base + s * C::STAGE_BYTES; };
    auto sB = [&](int s) { return smem_base + s * C::STAGE_BYTES + C::A_BYTES; };
    auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
    auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
    auto tfull_bar = [&](int b) { return smem_u32(&bars[2 * STAGES + b]); };
    auto tempty_bar = [&](int b) { return smem_u32(&bars[2 * STAGES + 2 + b]); };
    const uint32_t drain_bar = smem_u32(&bars[2 * STAGES + 4]);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (g.tma_store) prefetch_tmap(&tmC);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 2 * EPI_WARPS2);   // epilogue warps x 2 CTAs
        }
        mbar_init(drain_bar, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int mn_tiles = g.m_tiles * g.n_tiles;
    const int cluster_id = blockIdx.x >> 1;
    const int nclusters = gridDim.x >> 1;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            UnitIter ui;
            units_begin(g, cluster_id, nclusters, ui);
            Unit un;
            while (ok && units_next(g, mn_tiles, ui, un)) {
                const int mt = un.tile % g.m_tiles, nt = un.tile / g.m_tiles;
                const int kb1 = un.k1;
                for (int kb = un.k0; kb < kb1; ++kb) {
                    if (g.prefetch && kb + g.prefetch < kb1) {
                        tma_prefetch_2d(&tmA, (kb + g.prefetch) * BK_ELEMS, mt * 2 * BM + rank * BM);
                        tma_prefetch_2d(&tmB, (kb + g.prefetch) * BK_ELEMS, nt * BN + rank * C::BNH);
                    }
                    if (!mbar_wait(empty_bar(s), ph ^ 1, g.err, ERR_WAIT_PRODUCER)) { ok = false; break; }
                    const uint32_t lf = mapa_shared(full_bar(s), 0);
                    if (leader) mbar_arrive_expect_tx(full_bar(s), 2 * C::STAGE_BYTES);
                    tma_load_2d_pair(sA(s), &tmA, kb * BK_ELEMS, mt * 2 * BM + rank * BM, lf);
                    tma_load_2d_pair(sB(s), &tmB, kb * BK_ELEMS, nt * BN + rank * C::BNH, lf);
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // the whole warp runs the issue loop (warp-uniform addresses and
        // descriptors); one elected lane issues each tcgen05 instruction
        if (leader) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int it = 0;
            UnitIter ui;
            units_begin(g, cluster_id, nclusters, ui);
            Unit un;
            for (; ok && units_next(g, mn_tiles, ui, un); ++it) {
                const int b = it & 1;
                const uint32_t aph = (it >> 1) & 1;
                if (!mbar_wait_warp(tempty_bar(b), aph ^ 1, g.err, ERR_WAIT_MMA_ACC)) { ok = false; break; }
                tc_fence_after();
                const uint32_t dcol = tmem_base + b * BN;
                const int kb0 = un.k0, kb1 = un.k1;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait_warp(full_bar(s), ph, g.err, ERR_WAIT_MMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128(sA(s));
                    const uint64_t bdesc = smem_desc_sw128(sB(s));
                    if (elect_one()) {
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint64_t koff = static_cast<uint64_t>((k * 32) >> 4);
                            const uint32_t acc = (kb != kb0) || (k != 0);
                            if (KIND == RKB_IN_I8)        tc_mma_i8_pair(dcol, adesc + koff, bdesc + koff, IDESC, acc);
                            else if (KIND == RKB_IN_TF32) tc_mma_tf32_pair(dcol, adesc + koff, bdesc + koff, IDESC, acc);
                            else                          tc_mma_f16_pair(dcol, adesc + koff, bdesc + koff, IDESC, acc);
                        }
                        tc_commit_pair(empty_bar(s));
                        tc_commit_pair(mapa_shared(empty_bar(s), peer));
                    }
                    __syncwarp();
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                if (ok && elect_one()) {
                    tc_commit_pair(tfull_bar(b));
                    tc_commit_pair(mapa_shared(tfull_bar(b), peer));
                }
                __syncwarp();
            }
            if (!ok && elect_one()) {
                tc_commit_pair(drain_bar);
                mbar_wait_drain(drain_bar, 0);
            }
            __syncwarp();
        }
    } else {
        const int e = warp - 2;                  // epilogue warp 0..7
        const int q = warp & 3;                  // TMEM lane quarter
        const int c_lo = (e >> 2) * (BN / 2), c_hi = c_lo + BN / 2;   // this warp's columns
        int it = 0;
        uint32_t nstore = 0;
        const uint32_t lempty0 = mapa_shared(tempty_bar(0), 0);
        const uint32_t lempty1 = mapa_shared(tempty_bar(1), 0);
        UnitIter ui;
        units_begin(g, cluster_id, nclusters, ui);
        Unit un;
        for (; units_next(g, mn_tiles, ui, un); ++it) {
            const int b = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!mbar_wait_warp(tfull_bar(b), aph, g.err, ERR_WAIT_EPILOGUE)) break;
            tc_fence_after();
            const int mt = un.tile % g.m_tiles, nt = un.tile / g.m_tiles;
            const int row = mt * 2 * BM + rank * BM + q * 32 + lane;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * BN;
            Args gs = g;   // split-K partial slab of this unit
            if (g.k_splits > 1)
                gs.C = static_cast<float *>(g.C) + static_cast<long>(un.tl) * g.split_stride;
            // stream-K split segment: add the accumulator into the tile's sum buffer
            // (fire-and-forget reductions, exact in int32), release TMEM, count in;
            // the last of the tile's segments to arrive reads the sum and stores C
            bool from_sum = false;
            const uint32_t *sum_w = nullptr;
            if (un.split) {
                uint32_t *acc = static_cast<uint32_t *>(g.sk_part) +
                                (static_cast<size_t>(un.tl) * 2 * BM * BN) +
                                static_cast<size_t>(rank * 4 + q) * (BN / 32) * 1024 + lane;
#pragma unroll 1
                for (int c = c_lo; c < c_hi; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j) atomicAdd(acc + (c / 32) * 1024 + j * 32, r[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(b ? lempty1 : lempty0);
                const int kb = g.k_blocks;
                const int nseg = (un.tl * kb + kb - 1) / g.sk_L - (un.tl * kb) / g.sk_L + 1;
                int last = 0;
                if (lane == 0) {
                    __threadfence();
                    last = atomicAdd(g.sk_cnt + (un.tl * 2 + rank) * EPI_WARPS2 + e, 1) == nseg - 1;
                    if (last) __threadfence();
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) continue;
                from_sum = true;
                sum_w = acc;
            }
            // 32 words of this warp's rows for chunk c: from TMEM, or from the sum buffer
            auto load_chunk = [&](uint32_t (&r)[32], int c) {
                if (from_sum) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) r[j] = __ldcg(sum_w + (c / 32) * 1024 + j * 32);
                } else {
                    tmem_ld32(tbase + c, r);
                    tmem_ld_wait();
                }
            };
            if (g.tma_store) {
                const int row0 = row - lane;
#pragma unroll 1
                for (int c = c_lo; c < c_hi; c += 32) {
                    uint32_t r[32];
                    load_chunk(r, c);
                    if (c + 32 == c_hi && !from_sum) {   // accumulator drained: release it before the last store
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(b ? lempty1 : lempty0);
                    }
                    const int col = nt * BN + c;
                    if (col >= g.N) continue;
                    pack_chunk<OUT>(g, row, col, r);
                    // fp16 chunks are 2 KB: two buffers in the warp's 4 KB, else one
                    constexpr int NBUF = OUT == RKB_OUT_F16 ? 2 : 1;
                    const uint32_t buf = stg_base + e * 4096 + (nstore % NBUF) * (4096 / NBUF);
                    if (lane == 0) bulk_wait_read<NBUF - 1>();   // the store that used buf has read it
                    __syncwarp();
                    stage_store<OUT>(&tmC, buf, lane, r, col, row0, g.k_splits > 1 ? un.tl : -1);
                    ++nstore;
                }
                continue;
            }
#pragma unroll 1
            for (int c = c_lo; c < c_hi; c += 32) {
                uint32_t r[32];
                load_chunk(r, c);
                const int col = nt * BN + c;
                if (col < g.N) store_chunk<OUT>(gs, row, col, r);
            }
            if (from_sum) continue;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(b ? lempty1 : lempty0);
        }
        if (lane == 0 && g.tma_store) bulk_wait<0>();
    }

    tc_fence_before();
    __syncwarp();   // reconverge role-divergent lanes: the barrier below is warp-aligned
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    }
}



template <int KIND, int OUT, int BN>
int launch2(const rkb_gemm_desc *d, int *err, cudaStream_t stream, int splits = 1, int use_sk = 0) {
    using C = Cfg2<BN>;
    static std::once_flag attr_once[16];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 15], [] {
        cudaFuncSetAttribute(gemm2_kernel<KIND, OUT, BN>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    const int esize = Kind<KIND>::ESIZE;
    const CUtensorMapDataType dt = Kind<KIND>::DT;
    CUtensorMap ta, tb;
    if (make_tmap_2d(&ta, d->A, dt, esize, d->K, d->M, d->lda, BK_BYTES / esize, BM) ||
        make_tmap_2d(&tb, d->B, dt, esize, d->K, d->N, d->ldb, BK_BYTES / esize, C::BNH))
        return ROCKET_E_SHAPE;
    Args g;
    g.M = d->M; g.N = d->N; g.K = d->K;
    g.m_tiles = (d->M + 2 * BM - 1) / (2 * BM);
    g.n_tiles = (d->N + BN - 1) / BN;
    g.k_blocks = (d->K * esize + BK_BYTES - 1) / BK_BYTES;
    g.C = d->C; g.ldc = d->ldc;
    g.row_scale = d->row_scale; g.col_scale = d->col_scale;
    g.bias = static_cast<const __half *>(d->bias);
    g.residual = static_cast<const __half *>(d->residual);
    g.ldr = d->ldr; g.act = d->act;
    g.k_splits = splits;
    g.kb_per_split = (g.k_blocks + splits - 1) / splits;
    g.split_stride = static_cast<long>(d->M) * d->N;
    if (splits > 1) {   // fp32 partial slabs [splits][M][N], no epilogue extras
        g.C = d->workspace;
        g.ldc = d->N;
        g.row_scale = g.col_scale = nullptr;
        g.bias = g.residual = nullptr;
        g.act = RKB_ACT_NONE;
    }
    g.err = err;
    // staged TMA stores of C (not for split-K slabs: a tile past M would spill
    // into the next slab)
    CUtensorMap tc;
    if (splits == 1) {
        g.tma_store = c_store_map<OUT>(&tc, d->M, d->N, g.C, g.ldc, g.k_blocks,
                                       g.bias || g.residual || g.act != RKB_ACT_NONE);
    } else {   // fp32 partial slabs [splits][M][N]: a 3D map clips rows past M within each slab
        memset(&tc, 0, sizeof tc);
        g.tma_store = encode_tmap_3d(&tc, g.C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d->N, d->M, splits, d->N,
                                     static_cast<long>(d->M) * d->N, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B) == 0;
    }
    g.prefetch = prefetch_distance();
    const int tiles = g.m_tiles * g.n_tiles * splits;
    const int pairs = rkb_device_sm_count(dev) / 2;
    int grid = 2 * (tiles < pairs ? tiles : pairs);
    g.sk = 0; g.sk_W = g.sk_R = g.sk_L = 0; g.sk_part = nullptr; g.sk_cnt = nullptr;
    if (splits == 1 && use_sk && d->workspace) {
        const SkPlan sp = sk_plan(d->M, d->N, d->K, esize, BN, rkb_device_sm_count(dev));
        if (sp.on) {
            g.sk = 1; g.sk_W = sp.W; g.sk_R = sp.R; g.sk_L = sp.L;
            g.sk_part = d->workspace;
            g.sk_cnt = reinterpret_cast<int *>(static_cast<char *>(d->workspace) + sp.part_bytes);
            // sum buffers and arrival counters start at zero every launch
            if (cudaMemsetAsync(d->workspace, 0, sp.part_bytes + sp.cnt_bytes, stream) != cudaSuccess)
                return ROCKET_E_DEVICE;
            grid = 2 * sp.P;
        }
    }
    gemm2_kernel<KIND, OUT, BN><<<grid, NUM_THREADS2, C::SMEM, stream>>>(ta, tb, tc, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "rkb gemm2 launch: %s\n", cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    return 0;
}


// Kernel choice by estimated time: waves x (per-SM tile area x K-blocks) /
// assumed efficiency, over single-CTA tiles 128 x BN and CTA-pair tiles
// 256 x BN on two SMs.  A pair option whose last wave would run under-filled
// may instead take the stream-K tail (sk_plan): fractional waves plus a fixed
// cost for the zeroed sum buffers and the tail exchange (about 15 us, here
// in the same units: 1 unit ~ 11 ps on B200).  Efficiencies and the fixed
// cost were fitted to measured int8 GEMMs at the 12B-prefill shapes.
// Returns 0x100 | BN for the pair kernel, BN for the single-CTA one.
struct Pick { int code, sk; };
// process-wide override (rocket_b200_gemm_policy); 0 / -1 = automatic
inline std::atomic<int> &policy_variant() { static std::atomic<int> v{0}; return v; }
inline std::atomic<int> &policy_sk() { static std::atomic<int> v{-1}; return v; }
inline Pick pick_kernel(int M, int N, int K, int esize) {
    static const char *e = getenv("ROCKET_GEMM_VARIANT");
    const int kb = (K * esize + BK_BYTES - 1) / BK_BYTES;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = rkb_device_sm_count(dev);
    const int pv = policy_variant().load(std::memory_order_relaxed);
    const int psk = policy_sk().load(std::memory_order_relaxed);
    if (pv || e) {
        int v = pv ? pv : atoi(e);
        if (v == 384) v = 0x180;
        if (v == 512) v = 0x200;
        if (v == 128 || v == 256 || v == 0x180 || v == 0x200) {
            const int sk = (v & 0x100) && psk != 0 ? sk_plan(M, N, K, esize, v == 0x200 ? 256 : 128, sms).on : 0;
            return Pick{v, sk};
        }
    }
    constexpr double SK_FIXED = 1.3e6;
    struct Opt { int code, tm, bn, unit; double eff; } opts[] = {
        {256, 128, 256, 1, 0.66}, {128, 128, 128, 1, 0.60},
        {0x200, 256, 256, 2, 0.82}, {0x180, 256, 128, 2, 0.55}};
    double best = 1e300;
    Pick pk{256, 0};
    for (const Opt &o : opts) {
        const double tiles = std::ceil(M / double(o.tm)) * std::ceil(N / double(o.bn));
        const double units = sms / o.unit;
        const double tile_t = double(o.tm) * o.bn / o.unit * kb / o.eff;
        const double t_dp = std::ceil(tiles / units) * tile_t;
        if (t_dp < best * 0.999) { best = t_dp; pk = Pick{o.code, 0}; }
        if (o.unit == 2 && psk != 0 && sk_plan(M, N, K, esize, o.bn, sms).on) {
            const double t_sk = tiles / units * tile_t + SK_FIXED;
            if (t_sk < best * 0.999 || psk == 1) { best = t_sk; pk = Pick{o.code, 1}; }
        }
    }
    return pk;
}

// Split-K reduction: C = epilogue(sum over splits of the fp32 partials), the
// splits summed in index order (deterministic).  8 outputs per thread.
template <int OUT>
__global__ void split_reduce(const float *__restrict__ ws, int splits, long stride, int M, int N,
                             void *C, long ldc, const __half *bias, int act, const __half *res, long ldr) {
    const long n8 = static_cast<long>(M) * (N / 8);
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int row = static_cast<int>(i / (N / 8)), col = static_cast<int>(i % (N / 8)) * 8;
        float f[8];
        const float4 *p0 = reinterpret_cast<const float4 *>(ws + static_cast<long>(row) * N + col);
        float4 a = p0[0], b = p0[1];
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
        for (int s = 1; s < splits; ++s) {
            const float4 *p = reinterpret_cast<const float4 *>(ws + s * stride + static_cast<long>(row) * N + col);
            a = p[0]; b = p[1];
            f[0] += a.x; f[1] += a.y; f[2] += a.z; f[3] += a.w; f[4] += b.x; f[5] += b.y; f[6] += b.z; f[7] += b.w;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (bias) f[j] += __half2float(bias[col + j]);
            f[j] = apply_act(f[j], act);
            if (res) f[j] += __half2float(res[static_cast<long>(row) * ldr + col + j]);
        }
        if (OUT == RKB_OUT_F32) {
            float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(C) + static_cast<long>(row) * ldc + col);
            o[0] = make_float4(f[0], f[1], f[2], f[3]);
            o[1] = make_float4(f[4], f[5], f[6], f[7]);
        } else {
            uint32_t h[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                __half2 p = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
                h[j] = *reinterpret_cast<uint32_t *>(&p);
            }
            *reinterpret_cast<uint4 *>(static_cast<__half *>(C) + static_cast<long>(row) * ldc + col) =
                make_uint4(h[0], h[1], h[2], h[3]);
        }
    }
}

// Split count for fp16 inputs: split-K over the CTA-pair 256x256 kernel with
// fp32 partial slabs and a deterministic reduce (splits summed in index order).
// Automatic when the pair tiles cannot fill the GPU and K is long (at least 48
// K-blocks): splits = clamp(pairs / tiles, 2, 3).  Measured on B200, fp16
// 512x4096x4096: 35.3 -> 26.7 us; 256x4096x4096: 32.8 -> 21.0 us;
// 1024x4096x4096: 51 -> 43 us.  ROCKET_GEMM_SPLITK = 1..4 overrides (1 = off).
inline int pick_splits(const rkb_gemm_desc *d) {
    if (d->in_kind != RKB_IN_F16 || d->row_scale || d->col_scale) return 1;
    const int kblocks = (d->K * 2 + BK_BYTES - 1) / BK_BYTES;
    const char *e = getenv("ROCKET_GEMM_SPLITK");
    int s;
    if (e) {
        s = atoi(e);
        if (s > 4) s = 4;
    } else {
        int dev = 0;
        cudaGetDevice(&dev);
        const int pairs = rkb_device_sm_count(dev) / 2;
        const int tiles = ((d->M + 2 * BM - 1) / (2 * BM)) * ((d->N + 255) / 256);
        if (tiles >= pairs || kblocks < 48 || (d->N & 7)) return 1;
        s = pairs / tiles;
        s = s < 2 ? 2 : s > 3 ? 3 : s;
    }
    while (s > 1 && kblocks / s < 4) --s;
    return s < 1 ? 1 : s;
}

}  // namespace dense
}  // namespace rkb

extern "C" int rocket_b200_gemm_policy(int variant, int stream_k) {
    if (variant != 0 && variant != 128 && variant != 256 && variant != 384 && variant != 512) return ROCKET_E_SHAPE;
    if (stream_k < -1 || stream_k > 1) return ROCKET_E_SHAPE;
    rkb::dense::policy_variant().store(variant == 384 ? 0x180 : variant == 512 ? 0x200 : variant);
    rkb::dense::policy_sk().store(stream_k);
    return 0;
}

extern "C" int rkb_gemm_launches(const rkb_gemm_desc *d) {
    return rkb::dense::pick_splits(d) > 1 ? 2 : 1;   // split-K adds its reduce kernel
}

extern "C" size_t rkb_gemm_workspace_bytes(const rkb_gemm_desc *d) {
    using namespace rkb::dense;
    const int s = pick_splits(d);
    if (s > 1) return static_cast<size_t>(s) * d->M * d->N * sizeof(float);
    const int esize = d->in_kind == RKB_IN_I8 ? 1 : d->in_kind == RKB_IN_TF32 ? 4 : 2;
    const Pick pk = pick_kernel(d->M, d->N, d->K, esize);
    if (!pk.sk) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    const SkPlan sp = sk_plan(d->M, d->N, d->K, esize, pk.code == 0x200 ? 256 : 128, rkb_device_sm_count(dev));
    return sp.on ? sp.part_bytes + sp.cnt_bytes : 0;
}

extern "C" int rkb_gemm_run(const rkb_gemm_desc *d, int *err, cudaStream_t stream) {
    using namespace rkb::dense;
    if (d->M <= 0 || d->N <= 0 || d->K <= 0) return ROCKET_E_SHAPE;
    if ((d->N & 7) || (d->ldc & 7)) return ROCKET_E_SHAPE;
    const int splits = pick_splits(d);
    if (splits > 1) {
        if (!d->workspace || (d->N & 7)) return ROCKET_E_NOMEM;
        int rc = launch2<RKB_IN_F16, RKB_OUT_F32, 256>(d, err, stream, splits);
        if (rc) return rc;
        const long n8 = static_cast<long>(d->M) * (d->N / 8);
        int grid = static_cast<int>((n8 + 255) / 256);
        if (grid > 148 * 8) grid = 148 * 8;
        const long stride = static_cast<long>(d->M) * d->N;
        const __half *bias = static_cast<const __half *>(d->bias);
        const __half *res = static_cast<const __half *>(d->residual);
        if (d->out_kind == RKB_OUT_F16)
            split_reduce<RKB_OUT_F16><<<grid, 256, 0, stream>>>(static_cast<const float *>(d->workspace), splits,
                                                                 stride, d->M, d->N, d->C, d->ldc, bias, d->act, res, d->ldr);
        else
            split_reduce<RKB_OUT_F32><<<grid, 256, 0, stream>>>(static_cast<const float *>(d->workspace), splits,
                                                                 stride, d->M, d->N, d->C, d->ldc, bias, d->act, res, d->ldr);
        return cudaGetLastError() == cudaSuccess ? 0 : ROCKET_E_DEVICE;
    }
    const Pick pk = pick_kernel(d->M, d->N, d->K, d->in_kind == RKB_IN_I8 ? 1 : d->in_kind == RKB_IN_TF32 ? 4 : 2);
    const int v = pk.code;
#define RKB_DISPATCH(KIND, OUT)                                                   \
    switch (v) {                                                                  \
    case 0x200: return launch2<KIND, OUT, 256>(d, err, stream, 1, pk.sk);         \
    case 0x180: return launch2<KIND, OUT, 128>(d, err, stream, 1, pk.sk);         \
    case 128:   return launch<KIND, OUT, 128>(d, err, stream);                    \
    default:    return launch<KIND, OUT, 256>(d, err, stream);                    \
    }
    if (d->in_kind == RKB_IN_F16) {
        if (d->out_kind == RKB_OUT_F16) { RKB_DISPATCH(RKB_IN_F16, RKB_OUT_F16); }
        if (d->out_kind == RKB_OUT_F32) { RKB_DISPATCH(RKB_IN_F16, RKB_OUT_F32); }
    } else if (d->in_kind == RKB_IN_I8) {
        if (d->out_kind == RKB_OUT_I32) { RKB_DISPATCH(RKB_IN_I8, RKB_OUT_I32); }
    } else if (d->in_kind == RKB_IN_BF16) {
        if (d->out_kind == RKB_OUT_F32) { RKB_DISPATCH(RKB_IN_BF16, RKB_OUT_F32); }
    } else if (d->in_kind == RKB_IN_TF32) {
        if (d->out_kind == RKB_OUT_F32) { RKB_DISPATCH(RKB_IN_TF32, RKB_OUT_F32); }
    }
#undef RKB_DISPATCH
    return ROCKET_E_UNSUPPORTED;
}
