// wgemm_ts.cu -- group-wise quantised-weight GEMM with the dequantised weights
// fed to the tensor core from TMEM (tcgen05.mma with its A operand in tensor
// memory).
//
// Same contract as the MODE_F16 path of wgemm_tc.cu (reference group-wise
// entries: src/rocket_matmul.c:2716-2871 and :3132-3282, resident forms in
// src/rocket_prepacked_int8.c / _int4.c):
//     C[m, n] = row_scale[m] * sum_k A16[m, k] * (w[n, k] * s[n, k / 32])
// with the codes and fp16 scales in the resident tiled layout of rkb_wpack_*.
//
// Why TMEM: writing the dequantised tile to shared memory and reading it back
// through the MMA costs ~64 KB of shared-memory traffic per 64-wide K block on
// top of the TMA fills -- more than the SM's shared-memory bandwidth at the
// tensor rate.  Here each dequantising thread owns one weight row (one TMEM
// lane) and writes its 32 fp16 pairs with tcgen05.st, so the weights never
// touch shared memory after their 4 KB code block lands.
//
// The MMA computes C^T tiles: 128 weight rows (M, A operand in TMEM) against
// NT <= 384 tokens (B = activations, TMA-loaded, 128-byte swizzled), issued as
// two MMAs of N = NT / 2 <= 192 that share the dequantised A tile.  The cost
// that bounds this kernel is the dequantisation (about 2.25 instructions per
// weight on 8 warps), so the tile is made as wide in tokens as TMEM allows:
// every dequantised weight feeds NT MACs.  (At NT = 192 -- and equally with
// 256 weight rows per activation tile -- ncu showed the tensor pipe 40% busy
// with the dequant warps in fixed-latency waits.)  The accumulators take TMEM
// columns [0, 384) single-buffered; the A ring takes [384, 512).  NT is chosen
// per call to balance waves over the 148 SMs.  Roles (448 threads):
//   warp 0      producer: TMA activation tile (two boxes) + bulk copies of the
//               half code block and half scale block, RS-deep raw ring
//   warp 1      MMA issuer: per K block 2 x 4 MMAs (one per token half)
//   warps 2..5  epilogue: thread = weight row n, loops over tokens; every
//               store instruction writes 32 consecutive n of one token row
//   warps 6..13 dequantisers: warp (q, h) owns TMEM lanes 32q..32q+31 and the
//               h-th 32-code half of each K block; tcgen05.st into a DA-deep
//               TMEM ring of A tiles
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>
#include <cmath>

#include "rkb_ptx.cuh"
#include "rkb_tmap.h"
#include "rkb_wlayout.cuh"
#include "../src/rkb_kernels.h"
#include "../../include/rocket_npu.h"

namespace rkb {
namespace wts {

constexpr int WM = 128;           // weight rows per tile (MMA M)
constexpr int NH_MAX = 192;       // tokens per MMA (N); a tile is two of them
constexpr int NUM_THREADS = 448;
constexpr int DEQ_WARP0 = 6;
constexpr int DA = 4;             // TMEM A-ring depth (64-wide K blocks)
constexpr int ACOLS = 32;         // TMEM columns per A tile: 128 lanes x 64 fp16
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t A_COL0 = 2 * NH_MAX;   // accumulators in [0, 384), A ring after
static_assert(A_COL0 + DA * ACOLS <= TMEM_COLS, "TMEM budget");

template <int WBITS>
struct Cfg {
    static constexpr int B_BYTES = 2 * NH_MAX * 128;                  // activations, 64 fp16 per row
    static constexpr int CODE_BYTES = WM * 64 * WBITS / 8;            // half of a 256-row block
    static constexpr int SCALE_BYTES = WM * 2 * 2;
    static constexpr int RAW_BYTES = (B_BYTES + CODE_BYTES + SCALE_BYTES + 1023) / 1024 * 1024;
    static constexpr int RS = WBITS == 4 ? 4 : 3;
    static constexpr int NBARS = 2 * RS + 2 * DA + 3;
    static constexpr int SMEM = RS * RAW_BYTES + NBARS * 8 + 16 + 1024;
    static_assert(SMEM <= 232448, "shared memory budget");
};

struct Args {
    int M, N, K;
    int nh;                   // tokens per MMA (N); a tile covers 2 * nh tokens
    int m_tiles, n_tiles, k_blocks, kb64_total;
    const uint8_t *codes;     // resident tiled codes (256-row blocks)
    const __half *scales;     // resident tiled fp16 scales
    void *C;
    long ldc;
    const float *row_scale;
    int *err;
};

RKB_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
          "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
          "r"(r[14]), "r"(r[15])
        : "memory");
}
RKB_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D(tmem) (+)= A(tmem) * B(smem desc)^T, fp16 inputs, fp32 accumulate.
RKB_DEV void tc_mma_f16_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
        ::"r"(d), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accum) : "memory");
}

RKB_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
RKB_DEV uint32_t lop_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
RKB_DEV uint32_t h2_sub_mul(uint32_t x, uint32_t bias, uint32_t s2) {
    __half2 hx = *reinterpret_cast<__half2 *>(&x);
    __half2 hb = *reinterpret_cast<__half2 *>(&bias);
    __half2 hs = *reinterpret_cast<__half2 *>(&s2);
    __half2 r = __hmul2(__hsub2(hx, hb), hs);
    return *reinterpret_cast<uint32_t *>(&r);
}
// 8 offset-binary int4 codes -> 4 packed fp16 pairs (v * s), pair j = codes 2j, 2j+1
RKB_DEV void deq8_i4(uint32_t u, uint32_t s2, uint32_t *o) {
    const uint32_t e = u & 0x0F0F0F0Fu, od = (u >> 4) & 0x0F0F0F0Fu;
    o[0] = h2_sub_mul(lop_and_or(prmt(e, od, 0x4400u), 0x00FF00FFu, 0x64006400u), 0x64086408u, s2);
    o[1] = h2_sub_mul(lop_and_or(prmt(e, od, 0x5511u), 0x00FF00FFu, 0x64006400u), 0x64086408u, s2);
    o[2] = h2_sub_mul(lop_and_or(prmt(e, od, 0x6622u), 0x00FF00FFu, 0x64006400u), 0x64086408u, s2);
    o[3] = h2_sub_mul(lop_and_or(prmt(e, od, 0x7733u), 0x00FF00FFu, 0x64006400u), 0x64086408u, s2);
}
// 4 offset-binary int8 codes -> 2 packed fp16 pairs
RKB_DEV void deq4_i8(uint32_t w, uint32_t s2, uint32_t *o) {
    o[0] = h2_sub_mul(prmt(w, 0x64646464u, 0x5140u), 0x64806480u, s2);
    o[1] = h2_sub_mul(prmt(w, 0x64646464u, 0x7362u), 0x64806480u, s2);
}

template <int WBITS, int OUT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
wgemm_ts_kernel(const __grid_constant__ CUtensorMap tmB, const Args g) {
    using C = Cfg<WBITS>;
    constexpr int RS = C::RS;
    const int nh = g.nh, nt = 2 * nh;
    const int dstride = (nh + 31) & ~31;   // token half p at TMEM column p * dstride
    const uint32_t IDESC = idesc_f16_f32acc(WM, nh);
    constexpr int RB = 64 * WBITS / 8;               // code bytes per row of a 64-wide K block
    const int tx_b = nt * 128;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + RS * C::RAW_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBARS);
    const uint32_t sbase = smem_u32(smem);
    auto sB = [&](int r) { return sbase + r * C::RAW_BYTES; };
    auto sCode = [&](int r) { return sbase + r * C::RAW_BYTES + C::B_BYTES; };
    auto sScale = [&](int r) { return sCode(r) + C::CODE_BYTES; };
    auto pCode = [&](int r) { return smem + r * C::RAW_BYTES + C::B_BYTES; };
    auto pScale = [&](int r) {
        return reinterpret_cast<const uint16_t *>(smem + r * C::RAW_BYTES + C::B_BYTES + C::CODE_BYTES);
    };
    auto raw_full = [&](int r) { return smem_u32(&bars[r]); };
    auto raw_empty = [&](int r) { return smem_u32(&bars[RS + r]); };
    auto a_full = [&](int a) { return smem_u32(&bars[2 * RS + a]); };
    auto a_empty = [&](int a) { return smem_u32(&bars[2 * RS + DA + a]); };
    const uint32_t tfull_bar = smem_u32(&bars[2 * RS + 2 * DA]);
    const uint32_t tempty_bar = smem_u32(&bars[2 * RS + 2 * DA + 1]);
    const uint32_t drain_bar = smem_u32(&bars[2 * RS + 2 * DA + 2]);
    auto acol = [&](int a) { return A_COL0 + static_cast<uint32_t>(a * ACOLS); };
    auto sBh = [&](int r, int p) { return sB(r) + p * NH_MAX * 128; };   // token half p (1024-aligned)

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmB);
        for (int r = 0; r < RS; ++r) {
            mbar_init(raw_full(r), 1);
            mbar_init(raw_empty(r), 1);
        }
        for (int a = 0; a < DA; ++a) {
            mbar_init(a_full(a), 8);
            mbar_init(a_empty(a), 1);
        }
        mbar_init(tfull_bar, 1);
        mbar_init(tempty_bar, 4);
        mbar_init(drain_bar, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
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
                const int mt = t % g.m_tiles, nt128 = t / g.m_tiles;   // nt128: 128-row weight tile
                // half h of 256-row tile t256 in the ragged layout (rkb_wlayout.cuh):
                // rows past the weight's end are not stored and keep stale data
                const int t256 = nt128 >> 1, h = nt128 & 1;
                const int rows = wl_rows(g.N, t256);
                const int hv = rows - h * WM < WM ? rows - h * WM : WM;
                const uint32_t cbytes = static_cast<uint32_t>(hv * RB), sbytes = static_cast<uint32_t>(hv * 4);
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    if (!mbar_wait(raw_empty(r), ph ^ 1, g.err, ERR_WAIT_PRODUCER)) { ok = false; break; }
                    mbar_arrive_expect_tx(raw_full(r), tx_b + cbytes + sbytes);
                    tma_load_2d(sBh(r, 0), &tmB, kb * 64, mt * nt, raw_full(r));
                    tma_load_2d(sBh(r, 1), &tmB, kb * 64, mt * nt + nh, raw_full(r));
                    bulk_load(sCode(r), g.codes + wl_block(g.N, g.kb64_total, t256, kb, RB) + h * WM * RB,
                              cbytes, raw_full(r));
                    bulk_load(sScale(r),
                              reinterpret_cast<const uint8_t *>(g.scales) + wl_block(g.N, g.kb64_total, t256, kb, 4) + h * WM * 4,
                              sbytes, raw_full(r));
                    if (++r == RS) { r = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int r = 0, a = 0;
            uint32_t aph = 0;
            bool ok = true;
            int it = 0;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
                if (!mbar_wait(tempty_bar, (it & 1) ^ 1, g.err, ERR_WAIT_MMA_ACC)) { ok = false; break; }
                tc_fence_after();
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    // a_full(a) implies raw_full(r): the dequantisers waited for it
                    if (!mbar_wait(a_full(a), aph, g.err, ERR_WAIT_MMA_FULL)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int p = 0; p < 2; ++p) {
                        const uint64_t bdesc = smem_desc_sw128(sBh(r, p));
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            tc_mma_f16_ts(tmem_base + p * dstride, tmem_base + acol(a) + k * 8,
                                          bdesc + static_cast<uint64_t>(k * 2), IDESC, (kb | k) != 0);
                    }
                    tc_commit(raw_empty(r));
                    tc_commit(a_empty(a));
                    if (++r == RS) r = 0;
                    if (++a == DA) { a = 0; aph ^= 1; }
                }
                if (ok) tc_commit(tfull_bar);
            }
            if (!ok) {
                tc_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0);
            }
        }
    } else if (warp < DEQ_WARP0) {
        // epilogue: lane = weight row n; TMEM columns = tokens (half p at p * dstride)
        const int q = warp & 3;
        int it = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
            if (!mbar_wait_warp(tfull_bar, it & 1, g.err, ERR_WAIT_EPILOGUE)) break;
            tc_fence_after();
            const int mt = t % g.m_tiles, nt128 = t / g.m_tiles;
            const int n = nt128 * WM + q * 32 + lane;
#pragma unroll 1
            for (int p = 0; p < 2; ++p) {
                const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + p * dstride;
#pragma unroll 1
                for (int c = 0; c < nh; c += 32) {
                    uint32_t v[32];
                    tmem_ld32(tbase + c, v);
                    tmem_ld_wait();
                    const int m0 = mt * nt + p * nh + c;
                    // the chunk's 32 token scales: lane j loads token m0 + j, then broadcast
                    const int mj = m0 + lane;
                    const float rs_l = (g.row_scale && mj < g.M && c + lane < nh) ? __ldg(g.row_scale + mj) : 1.0f;
                    const bool full = c + 32 <= nh && m0 + 32 <= g.M && n < g.N;
                    if (full) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float x = __uint_as_float(v[j]) * __shfl_sync(0xffffffffu, rs_l, j);
                            const long off = static_cast<long>(m0 + j) * g.ldc + n;
                            if (OUT == RKB_OUT_F32) static_cast<float *>(g.C)[off] = x;
                            else static_cast<__half *>(g.C)[off] = __float2half_rn(x);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float sj = __shfl_sync(0xffffffffu, rs_l, j);
                            const int m = m0 + j;
                            if (c + j < nh && m < g.M && n < g.N) {
                                const float x = __uint_as_float(v[j]) * sj;
                                if (OUT == RKB_OUT_F32)
                                    static_cast<float *>(g.C)[static_cast<long>(m) * g.ldc + n] = x;
                                else
                                    static_cast<__half *>(g.C)[static_cast<long>(m) * g.ldc + n] = __float2half_rn(x);
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar);
        }
    } else {
        // dequantisers: warp (q, h): TMEM lanes 32q..+31 = weight rows, K half h
        const int dw = warp - DEQ_WARP0;
        const int q = warp & 3, h = dw >> 2;
        const int row = q * 32 + lane;
        int r = 0, a = 0;
        uint32_t rph = 0, aph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < g.k_blocks; ++kb) {
                if (!mbar_wait_warp(raw_full(r), rph, g.err, ERR_WAIT_DEQUANT) ||
                    !mbar_wait_warp(a_empty(a), aph ^ 1, g.err, ERR_WAIT_DEQUANT)) { ok = false; break; }
                const uint16_t sh = pScale(r)[row * 2 + h];
                const uint32_t s2 = static_cast<uint32_t>(sh) | (static_cast<uint32_t>(sh) << 16);
                uint32_t o[16];
                if (WBITS == 4) {
                    const uint4 u = *reinterpret_cast<const uint4 *>(pCode(r) + row * 32 + h * 16);
                    deq8_i4(u.x, s2, o + 0);
                    deq8_i4(u.y, s2, o + 4);
                    deq8_i4(u.z, s2, o + 8);
                    deq8_i4(u.w, s2, o + 12);
                } else {
                    const uint4 u0 = *reinterpret_cast<const uint4 *>(pCode(r) + row * 64 + h * 32);
                    const uint4 u1 = *reinterpret_cast<const uint4 *>(pCode(r) + row * 64 + h * 32 + 16);
                    deq4_i8(u0.x, s2, o + 0);  deq4_i8(u0.y, s2, o + 2);
                    deq4_i8(u0.z, s2, o + 4);  deq4_i8(u0.w, s2, o + 6);
                    deq4_i8(u1.x, s2, o + 8);  deq4_i8(u1.y, s2, o + 10);
                    deq4_i8(u1.z, s2, o + 12); deq4_i8(u1.w, s2, o + 14);
                }
                tmem_st16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acol(a) + h * 16, o);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full(a));
                if (++r == RS) { r = 0; rph ^= 1; }
                if (++a == DA) { a = 0; aph ^= 1; }
            }
        }
    }

    tc_fence_before();
    __syncwarp();   // reconverge role-divergent lanes: the barrier below is warp-aligned
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Tokens per MMA nh (a tile is 2 * nh tokens): the multiple of 16 (<= 192)
// that minimises waves x (2 * nh + 32) over the SMs; small M takes the least
// nh that covers it.
inline int pick_nh(int M, int n_tiles, int sms) {
    if (M <= 2 * NH_MAX) {
        const int nh = ((M + 1) / 2 + 15) / 16 * 16;
        return nh < 16 ? 16 : nh;
    }
    int best = NH_MAX;
    double best_t = 1e300;
    for (int nh = NH_MAX; nh >= 96; nh -= 16) {
        const double tiles = std::ceil(M / double(2 * nh)) * n_tiles;
        const double t = std::ceil(tiles / sms) * (2 * nh + 32);
        if (t < best_t * 0.999) { best_t = t; best = nh; }
    }
    return best;
}

template <int WBITS, int OUT>
int launch(const rkb_wgemm_desc *d, int *err, cudaStream_t stream) {
    using C = Cfg<WBITS>;
    static std::once_flag attr_once[16];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 15], [] {
        cudaFuncSetAttribute(wgemm_ts_kernel<WBITS, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    const int sms = rkb_device_sm_count(dev);
    Args g;
    g.M = d->M; g.N = d->N; g.K = d->K;
    g.n_tiles = (d->N + WM - 1) / WM;
    g.nh = pick_nh(d->M, g.n_tiles, sms);
    g.m_tiles = (d->M + 2 * g.nh - 1) / (2 * g.nh);
    CUtensorMap tb;
    if (make_tmap_2d(&tb, d->A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, d->K, d->M, d->lda, 64, g.nh))
        return ROCKET_E_SHAPE;
    const int kp = (d->K + 127) / 128 * 128;
    g.kb64_total = kp / 64;
    g.k_blocks = kp / 64;
    g.codes = static_cast<const uint8_t *>(d->Wq);
    g.scales = static_cast<const __half *>(d->Ws);
    g.C = d->C; g.ldc = d->ldc;
    g.row_scale = d->row_scale;
    g.err = err;
    const int tiles = g.m_tiles * g.n_tiles;
    const int grid = tiles < sms ? tiles : sms;
    wgemm_ts_kernel<WBITS, OUT><<<grid, NUM_THREADS, C::SMEM, stream>>>(tb, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "rkb wgemm_ts launch: %s\n", cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    return 0;
}

}  // namespace wts
}  // namespace rkb

// Entry for the fp16-activation group-wise path (a_f16 != 0).
extern "C" int rkb_wgemm_ts_run(const rkb_wgemm_desc *d, int *err, cudaStream_t stream) {
    using namespace rkb::wts;
    if (d->M <= 0 || d->N <= 0 || d->K <= 0 || !d->a_f16) return ROCKET_E_SHAPE;
    if (d->w_bits == 4) {
        if (d->out_kind == RKB_OUT_F32) return launch<4, RKB_OUT_F32>(d, err, stream);
        if (d->out_kind == RKB_OUT_F16) return launch<4, RKB_OUT_F16>(d, err, stream);
    } else if (d->w_bits == 8) {
        if (d->out_kind == RKB_OUT_F32) return launch<8, RKB_OUT_F32>(d, err, stream);
        if (d->out_kind == RKB_OUT_F16) return launch<8, RKB_OUT_F16>(d, err, stream);
    }
    return ROCKET_E_UNSUPPORTED;
}
