// wgemm_xi.cu -- precise group-wise quantised-weight GEMM on the int8 tensor
// cores: exact int32 partials per quantisation group.
//
// The reference defines the group-wise product as exact integer inner
// products per K group, scaled and summed in fp32
// (src/rocket_matmul.c:2842-2856, src/rocket_prepacked_int8.c:620-632):
//     C[m, n] = sum_g a_scale[m, g] * b_scale[n, g] * P_g[m, n],
//     P_g[m, n] = sum_{k in group g} A[m, k] * W[n, k]      (integers)
// and its gates hold the result to 1e-5 of the output rms against an fp64
// evaluation (tests/matmul_int8_groupwise_rocket.c:59-82).
//
//   * the int8 activations are read by TMA as they are (no conversion pass);
//   * dequantiser warps turn the resident weight codes (int4 nibbles or
//     offset int8 bytes) into signed int8 in a 128-byte-swizzled shared tile;
//   * tcgen05.mma kind::i8 sums one group into an int32 TMEM partial -- exact
//     for any group (|a w| <= 2^14, so 2^17 products fit int32);
//   * the epilogue converts each partial to fp32 (the reference's own
//     int -> float step; exact below 2^24) and accumulates b_scale[n, g] * P (times a_scale[m, g] when that varies
//     with g) in fp32 registers, in group order.
//
// Tiles are C^T: 128 weight rows (MMA M, one weight row per TMEM lane) x NT
// tokens (MMA N).  K advances in blocks of 128 (one 128-byte swizzle row).
// TMEM: 512 / NT partial buffers of NT int32 columns, so the MMAs of later
// groups run while a group is drained.  Roles:
//   warp 0      producer: TMA activation tile + bulk copies of two 64-wide
//               code blocks (rkb_wlayout.cuh)
//   warp 1      MMA issuer: one K = 32 MMA per 32 columns of K, a commit at
//               every group end
//   warps 2..3  dequantisers: thread = weight rows r and r + 64, 128 codes ->
//               128 signed bytes each, 16-byte swizzled stores
//   warps 4..   epilogue: warp (q, j) owns TMEM lanes 32q.. (weight rows) and
//               token columns 64j..64j+63; 64 fp32 running sums per thread;
//               every store instruction writes 32 consecutive n of one token
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>

#include "rkb_ptx.cuh"
#include "rkb_tmap.h"
#include "rkb_wlayout.cuh"
#include "../src/rkb_kernels.h"
#include "../../include/rocket_npu.h"

namespace rkb {
namespace wxi {

constexpr int WM = 128;                 // weight rows per tile (MMA M)
constexpr int NUM_DEQ = 2;              // 16 warps in all at NT = 192: 128 registers a thread
constexpr int DEQ_WARP0 = 2;
constexpr int EPI_WARP0 = DEQ_WARP0 + NUM_DEQ;
constexpr int W_BYTES = WM * 128;       // one signed int8 weight tile, 128 K

template <int WBITS, int NT>
struct Cfg {
    static constexpr int NUM_EPI = 4 * (NT / 64);
    static constexpr int NUM_THREADS = 32 * (EPI_WARP0 + NUM_EPI);
    static constexpr int B_BYTES = NT * 128;                        // activations, 128 K
    static constexpr int CB = WM * 64 * WBITS / 8;                  // one 64-wide code block
    static constexpr int RAW_BYTES = (B_BYTES + 2 * CB + 1023) / 1024 * 1024;
    static constexpr int RS = WBITS == 4 ? 4 : 3;                   // raw ring depth
    static constexpr int DS = 4;                                    // weight-tile ring depth
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int NB = 512 / NT;                             // partial buffers in TMEM
    static constexpr int NBARS = 2 * RS + 2 * DS + 2 * NB + 1;
    static constexpr int SMEM = RS * RAW_BYTES + DS * W_BYTES + NBARS * 8 + 16 + 1024;
    static_assert(NT % 64 == 0 && NT <= 256, "token tile");
    static_assert(SMEM <= 232448, "shared memory budget");
};

struct Args {
    int M, N, K;
    int m_tiles, n_tiles, k_blocks, kb64_total;
    int group, nG;
    const uint8_t *codes;       // resident tiled codes (256-row blocks)
    const float *b_scale;       // fp32 [N, nG]
    const float *a_scale_t;     // fp32 [nG, M] when a_scale varies with g, else NULL
    const float *row_scale;     // fp32 [M] applied at the end, or NULL
    void *C;
    long ldc;
    int *err;
};

// 4 offset-by-8 nibble pairs (even k low) -> 8 signed bytes in k order
RKB_DEV uint2 widen8_i4(uint32_t u) {
    // (x + 0x78) ^ 0x80 maps a code x in [0, 15] to the byte of x - 8
    const uint32_t e = ((u & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
    const uint32_t o = (((u >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
    uint32_t lo, hi;
    asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(lo) : "r"(e), "r"(o));
    asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(hi) : "r"(e), "r"(o));
    return make_uint2(lo, hi);
}

constexpr int XCH = 16;                 // partial columns per tcgen05.ld in the epilogue

RKB_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

RKB_DEV void tmem_ld(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld16(taddr, r); }

RKB_DEV void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

template <int WBITS, int NT, int OUT, bool AS_COL>
__global__ void __launch_bounds__(Cfg<WBITS, NT>::NUM_THREADS, 1)
wgemm_xi_kernel(const __grid_constant__ CUtensorMap tmB, const Args g) {
    using C = Cfg<WBITS, NT>;
    constexpr int RS = C::RS, DS = C::DS, NUM_EPI = C::NUM_EPI, NB = C::NB;
    constexpr int RB = 64 * WBITS / 8;               // code bytes per row of a 64-wide K block
    constexpr uint32_t IDESC = idesc_s8_s32acc(WM, NT);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + RS * C::RAW_BYTES + DS * W_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBARS);
    const uint32_t sbase = smem_u32(smem);
    auto sB = [&](int r) { return sbase + r * C::RAW_BYTES; };
    auto sCode = [&](int r) { return sbase + r * C::RAW_BYTES + C::B_BYTES; };
    auto pCode = [&](int r) { return smem + r * C::RAW_BYTES + C::B_BYTES; };
    auto sW = [&](int d) { return sbase + RS * C::RAW_BYTES + d * W_BYTES; };
    auto raw_full = [&](int r) { return smem_u32(&bars[r]); };
    auto raw_empty = [&](int r) { return smem_u32(&bars[RS + r]); };
    auto w_full = [&](int d) { return smem_u32(&bars[2 * RS + d]); };
    auto w_empty = [&](int d) { return smem_u32(&bars[2 * RS + DS + d]); };
    auto p_full = [&](int b) { return smem_u32(&bars[2 * RS + 2 * DS + b]); };
    auto p_empty = [&](int b) { return smem_u32(&bars[2 * RS + 2 * DS + NB + b]); };
    const uint32_t drain_bar = smem_u32(&bars[2 * RS + 2 * DS + 2 * NB]);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmB);
        for (int r = 0; r < RS; ++r) {
            mbar_init(raw_full(r), 1);
            mbar_init(raw_empty(r), 1);
        }
        for (int d = 0; d < DS; ++d) {
            mbar_init(w_full(d), NUM_DEQ);
            mbar_init(w_empty(d), 1);
        }
        for (int b = 0; b < NB; ++b) {
            mbar_init(p_full(b), 1);
            mbar_init(p_empty(b), NUM_EPI);
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
    const int grp_steps = g.group / 32;          // MMAs (K = 32) per group
    const int k_steps = g.K / 32;                // K % 32 == 0: the padded tail is never issued

    if (warp == 0) {
        if (lane == 0) {
            int r = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int mt = t % g.m_tiles, nt128 = t / g.m_tiles;
                // half h of 256-row tile t256 in the ragged layout: rows past
                // the weight's end are not stored and keep stale data
                const int t256 = nt128 >> 1, h = nt128 & 1;
                const int rows = wl_rows(g.N, t256);
                const int hv = rows - h * WM < WM ? rows - h * WM : WM;
                const uint32_t cbytes = static_cast<uint32_t>(hv * RB);
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    if (!mbar_wait(raw_empty(r), ph ^ 1, g.err, ERR_WAIT_PRODUCER)) { ok = false; break; }
                    mbar_arrive_expect_tx(raw_full(r), NT * 128 + 2 * cbytes);
                    tma_load_2d(sB(r), &tmB, kb * 128, mt * NT, raw_full(r));
#pragma unroll
                    for (int i = 0; i < 2; ++i)
                        bulk_load(sCode(r) + i * C::CB,
                                  g.codes + wl_block(g.N, g.kb64_total, t256, 2 * kb + i, RB) + h * WM * RB,
                                  cbytes, raw_full(r));
                    if (++r == RS) { r = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int r = 0, d = 0;
            uint32_t dph = 0;
            uint32_t s = 0;            // groups issued by this CTA (P buffer s % NB)
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                for (int kb = 0; kb < g.k_blocks && ok; ++kb) {
                    // w_full(d) implies raw_full(r): the dequantisers waited for it
                    if (!mbar_wait(w_full(d), dph, g.err, ERR_WAIT_MMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128(sW(d));
                    const uint64_t bdesc = smem_desc_sw128(sB(r));
#pragma unroll 1
                    for (int k = 0; k < 4; ++k) {
                        const int ks = kb * 4 + k;
                        if (ks >= k_steps) break;
                        const int pos = ks % grp_steps;
                        const uint32_t b = s % NB;
                        if (pos == 0) {
                            // the epilogue's arrive of use (s / NB) - 1 (or its initial one)
                            if (!mbar_wait(p_empty(b), (s / NB) & 1, g.err, ERR_WAIT_MMA_ACC)) { ok = false; break; }
                            tc_fence_after();
                        }
                        tc_mma_i8(tmem_base + b * NT, adesc + static_cast<uint64_t>(k * 2),
                                  bdesc + static_cast<uint64_t>(k * 2), IDESC, pos != 0);
                        if (pos == grp_steps - 1) {
                            tc_commit(p_full(b));
                            ++s;
                        }
                    }
                    tc_commit(raw_empty(r));
                    tc_commit(w_empty(d));
                    if (++r == RS) r = 0;
                    if (++d == DS) { d = 0; dph ^= 1; }
                }
            }
            if (!ok) {
                tc_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0);
            }
        }
    } else if (warp < EPI_WARP0) {
        // dequantisers: each thread converts weight rows of the tile
        int r = 0, d = 0;
        uint32_t rph = 0, dph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < g.k_blocks; ++kb) {
                if (!mbar_wait_warp(raw_full(r), rph, g.err, ERR_WAIT_DEQUANT) ||
                    !mbar_wait_warp(w_empty(d), dph ^ 1, g.err, ERR_WAIT_DEQUANT)) { ok = false; break; }
#pragma unroll
                for (int rr = 0; rr < WM / (32 * NUM_DEQ); ++rr) {
                    const int row = (rr * NUM_DEQ + warp - DEQ_WARP0) * 32 + lane;
                    const uint32_t xr = static_cast<uint32_t>(row & 7);
                    const uint32_t dst = sW(d) + row * 128;
#pragma unroll
                    for (int i = 0; i < 2; ++i) {       // the two 64-wide code blocks
                        if (WBITS == 4) {
                            const uint4 *src = reinterpret_cast<const uint4 *>(pCode(r) + i * C::CB + row * 32);
#pragma unroll
                            for (int v = 0; v < 2; ++v) {
                                const uint4 u = src[v];
                                const uint2 a0 = widen8_i4(u.x), a1 = widen8_i4(u.y);
                                const uint2 a2 = widen8_i4(u.z), a3 = widen8_i4(u.w);
                                const uint32_t c0 = static_cast<uint32_t>(i * 4 + v * 2);
                                st_shared_v4(dst + ((c0 ^ xr) << 4), a0.x, a0.y, a1.x, a1.y);
                                st_shared_v4(dst + (((c0 + 1) ^ xr) << 4), a2.x, a2.y, a3.x, a3.y);
                            }
                        } else {
                            const uint4 *src = reinterpret_cast<const uint4 *>(pCode(r) + i * C::CB + row * 64);
#pragma unroll
                            for (int v = 0; v < 4; ++v) {
                                const uint4 u = src[v];
                                const uint32_t c = static_cast<uint32_t>(i * 4 + v);
                                st_shared_v4(dst + ((c ^ xr) << 4), u.x ^ 0x80808080u, u.y ^ 0x80808080u,
                                             u.z ^ 0x80808080u, u.w ^ 0x80808080u);
                            }
                        }
                    }
                }
                fence_proxy_async_smem();   // generic-proxy stores -> visible to the MMA
                __syncwarp();
                if (lane == 0) mbar_arrive(w_full(d));
                if (++r == RS) { r = 0; rph ^= 1; }
                if (++d == DS) { d = 0; dph ^= 1; }
            }
        }
    } else {
        // epilogue: lane = weight row n; token columns 64j..64j+63 of the tile
        const int e = warp - EPI_WARP0;
        const int q = warp & 3, j = e >> 2;
        const uint32_t tl = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + j * 64;
        const int nseg = g.K / g.group;
        // every partial buffer starts free: the MMA's first wait on each
        // completes on this arrive
        if (lane == 0)
            for (int b = 0; b < NB; ++b) mbar_arrive(p_empty(b));
        uint32_t s = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            const int mt = t % g.m_tiles, nt128 = t / g.m_tiles;
            const int n = nt128 * WM + q * 32 + lane;
            const int m0 = mt * NT + j * 64;
            const bool n_ok = n < g.N;
            const float *bsrow = g.b_scale + static_cast<size_t>(n_ok ? n : 0) * g.nG;
            float acc[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) acc[c] = 0.f;
            // scales are loaded two groups ahead: an L2 round trip per group
            // would otherwise sit on the epilogue's critical path
            auto ld_bs = [&](int gi) { return (n_ok && gi < nseg) ? __ldg(bsrow + gi) : 0.f; };
            auto ld_as = [&](int gi, int off) {
                return (AS_COL && gi < nseg && m0 + off + lane < g.M)
                           ? __ldg(g.a_scale_t + static_cast<size_t>(gi) * g.M + m0 + off + lane) : 0.f;
            };
            float bs_n1 = ld_bs(0), bs_n2 = ld_bs(1);
            float as0_n1 = ld_as(0, 0), as1_n1 = ld_as(0, 32), as0_n2 = ld_as(1, 0), as1_n2 = ld_as(1, 32);
            for (int grp = 0; grp < nseg; ++grp, ++s) {
                const float bs = bs_n1, as0 = as0_n1, as1 = as1_n1;
                bs_n1 = bs_n2; as0_n1 = as0_n2; as1_n1 = as1_n2;
                bs_n2 = ld_bs(grp + 2);
                if (AS_COL) { as0_n2 = ld_as(grp + 2, 0); as1_n2 = ld_as(grp + 2, 32); }
                const uint32_t b = s % NB;
                if (!mbar_wait_warp(p_full(b), (s / NB) & 1, g.err, ERR_WAIT_EPILOGUE)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int h = 0; h < 64 / XCH; ++h) {
                    uint32_t v[XCH];
                    const uint32_t ta = tl + b * NT + h * XCH;
                    tmem_ld(ta, v);
                    tmem_ld_wait();
                    if (h == 64 / XCH - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(p_empty(b));
                    }
                    float *ac = acc + h * XCH;
                    const float2 bs2 = make_float2(bs, bs);
                    const float asl = h * XCH < 32 ? as0 : as1;
#pragma unroll
                    for (int c = 0; c < XCH; c += 2) {
                        // exact below 2^24, else rounded once as the reference's (float) cast
                        const float2 x = make_float2(__int2float_rn(static_cast<int>(v[c])),
                                                     __int2float_rn(static_cast<int>(v[c + 1])));
                        if (AS_COL) {
                            const int cc = (h * XCH + c) & 31;
                            ac[c] = fmaf(bs * __shfl_sync(0xffffffffu, asl, cc), x.x, ac[c]);
                            ac[c + 1] = fmaf(bs * __shfl_sync(0xffffffffu, asl, cc + 1), x.y, ac[c + 1]);
                        } else {
                            const float2 y = __ffma2_rn(bs2, x, make_float2(ac[c], ac[c + 1]));
                            ac[c] = y.x;
                            ac[c + 1] = y.y;
                        }
                    }
                }
            }
            if (!ok) break;
            // the chunk's token scales: lane c loads token m0 + c (+32), then broadcast
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int mh = m0 + h * 32;
                const float rs_l = (g.row_scale && mh + lane < g.M) ? __ldg(g.row_scale + mh + lane) : 1.0f;
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float x = acc[h * 32 + c] * __shfl_sync(0xffffffffu, rs_l, c);
                    const int m = mh + c;
                    if (m < g.M && n_ok) {
                        const long off = static_cast<long>(m) * g.ldc + n;
                        if (OUT == RKB_OUT_F32) static_cast<float *>(g.C)[off] = x;
                        else static_cast<__half *>(g.C)[off] = __float2half_rn(x);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncwarp();   // reconverge role-divergent lanes: the barrier below is warp-aligned
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

template <int WBITS, int NT, int OUT, bool AS_COL>
int launch(const rkb_wgemm_desc *d, int *err, cudaStream_t stream) {
    using C = Cfg<WBITS, NT>;
    static std::once_flag attr_once[16];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 15], [] {
        cudaFuncSetAttribute(wgemm_xi_kernel<WBITS, NT, OUT, AS_COL>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    const int sms = rkb_device_sm_count(dev);
    Args g;
    g.M = d->M; g.N = d->N; g.K = d->K;
    g.n_tiles = (d->N + WM - 1) / WM;
    g.m_tiles = (d->M + NT - 1) / NT;
    CUtensorMap tb;
    if (make_tmap_2d(&tb, d->A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, d->K, d->M, d->lda, 128, NT))
        return ROCKET_E_SHAPE;
    const int kp = (d->K + 127) / 128 * 128;
    g.kb64_total = kp / 64;
    g.k_blocks = kp / 128;
    g.group = d->group;
    g.nG = d->K / d->group;
    g.codes = static_cast<const uint8_t *>(d->Wq);
    g.b_scale = d->b_scale;
    g.a_scale_t = d->a_scale_t;
    g.row_scale = d->row_scale;
    g.C = d->C; g.ldc = d->ldc;
    g.err = err;
    const int tiles = g.m_tiles * g.n_tiles;
    const int grid = tiles < sms ? tiles : sms;
    wgemm_xi_kernel<WBITS, NT, OUT, AS_COL><<<grid, C::NUM_THREADS, C::SMEM, stream>>>(tb, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "rkb wgemm_xi launch: %s\n", cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    return 0;
}

}  // namespace wxi
}  // namespace rkb

#ifndef RKB_XI_NT
#define RKB_XI_NT 192
#endif

extern "C" int rkb_wgemm_xi_run(const rkb_wgemm_desc *d, int *err, cudaStream_t stream) {
    using namespace rkb::wxi;
    if (d->M <= 0 || d->N <= 0 || d->K <= 0 || d->K % 32 || d->a_f16 || !d->b_scale ||
        d->group <= 0 || d->group % 32 || d->K % d->group || d->lda % 16)
        return ROCKET_E_SHAPE;
#define RKB_XI(BITS, OUT)                                                          \
    return d->a_scale_t ? launch<BITS, RKB_XI_NT, OUT, true>(d, err, stream)       \
                        : launch<BITS, RKB_XI_NT, OUT, false>(d, err, stream)
    if (d->w_bits == 4) {
        if (d->out_kind == RKB_OUT_F32) { RKB_XI(4, RKB_OUT_F32); }
        if (d->out_kind == RKB_OUT_F16) { RKB_XI(4, RKB_OUT_F16); }
    } else if (d->w_bits == 8) {
        if (d->out_kind == RKB_OUT_F32) { RKB_XI(8, RKB_OUT_F32); }
        if (d->out_kind == RKB_OUT_F16) { RKB_XI(8, RKB_OUT_F16); }
    }
#undef RKB_XI
    return ROCKET_E_UNSUPPORTED;
}
