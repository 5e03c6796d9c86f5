// wgemm_xp.cu -- group-wise quantised-weight GEMM with exact integer partials
// per quantisation group ("precise" group-wise mode).
//
// The reference defines the group-wise product as exact integer inner
// products per K group, scaled and summed in fp32
// (src/rocket_matmul.c:2842-2856, src/rocket_prepacked_int8.c:620-632):
//     C[m, n] = sum_g a_scale[m, g] * b_scale[n, g] * P_g[m, n],
//     P_g[m, n] = sum_{k in group g} A[m, k] * W[n, k]      (integers)
// and its gates hold the result to 1e-5 of the output rms against an fp64
// evaluation (tests/matmul_int8_groupwise_rocket.c:59-82).  This kernel keeps
// that structure instead of multiplying the scales into fp16 operands:
//
//   * the weight codes are widened to fp16 WITHOUT a scale (integers up to
//     128 in magnitude are exact in fp16), and so are the int8 activations;
//   * the MMA (kind::f16, fp32 accumulate) sums one segment of K -- one group,
//     or a piece of at most 1024 when a wide int8 group could pass 2^24 -- so
//     the segment's partial is an exact integer held in fp32;
//   * the epilogue reads each segment's partial from TMEM and accumulates
//     b_scale[n, g] * P (times a_scale[m, g] when that varies with g) in fp32
//     registers, in group order.
// The only roundings are the fp32 products and sums across groups, as in the
// reference's own host accumulation.
//
// Tiles are C^T: 128 weight rows (MMA M, A operand in TMEM, one weight row per
// TMEM lane) x 128 tokens (MMA N, activations TMA-loaded with the 128-byte
// swizzle).  TMEM: partial buffers P0 [0,128) and P1 [128,256), double
// buffered so the MMAs of segment s+1 run while segment s is drained; the
// dequantised A ring takes [256, 512).  Roles (704 threads):
//   warp 0      producer: TMA activation tile + bulk copy of the half code block
//   warp 1      MMA issuer: 4 MMAs (K = 16) per 64-wide K block, a commit at
//               every segment end
//   warps 2..5  dequantisers: warp q owns TMEM lanes 32q..32q+31 (weight rows)
//               and widens each row's 64 codes to fp16 with byte permutes,
//               tcgen05.st into the A ring
//   warps 6..21 epilogue: warp (q, j) owns lanes 32q.. and token columns
//               32j..32j+31; 32 fp32 running sums per thread; every store
//               instruction writes 32 consecutive n of one token row
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
namespace wxp {

constexpr int WM = 128;                 // weight rows per tile (MMA M)
constexpr int NT = 128;                 // tokens per tile (MMA N)
constexpr int NUM_DEQ = 4;
constexpr int NUM_EPI = 16;
constexpr int DEQ_WARP0 = 2;
constexpr int EPI_WARP0 = DEQ_WARP0 + NUM_DEQ;
constexpr int NUM_THREADS = 32 * (EPI_WARP0 + NUM_EPI);
constexpr int DA = 8;                   // TMEM A-ring depth (64-wide K blocks)
constexpr int ACOLS = 32;               // TMEM columns per A tile: 128 lanes x 64 fp16
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t A_COL0 = 2 * NT;
static_assert(A_COL0 + DA * ACOLS <= TMEM_COLS, "TMEM budget");

template <int WBITS>
struct Cfg {
    static constexpr int B_BYTES = NT * 128;                         // activations, 64 fp16 per row
    static constexpr int CODE_BYTES = WM * 64 * WBITS / 8;           // half of a 256-row block
    static constexpr int RAW_BYTES = (B_BYTES + CODE_BYTES + 1023) / 1024 * 1024;
    static constexpr int RS = WBITS == 4 ? 8 : 7;
    static constexpr int NBARS = 2 * RS + 2 * DA + 5;
    static constexpr int SMEM = RS * RAW_BYTES + NBARS * 8 + 16 + 1024;
    static_assert(SMEM <= 232448, "shared memory budget");
};

struct Args {
    int M, N, K;
    int m_tiles, n_tiles, k_blocks, kb64_total;
    int group, seg, nG;
    const uint8_t *codes;       // resident tiled codes (256-row blocks)
    const float *b_scale;       // fp32 [N, nG] (this slice)
    const float *a_scale_t;     // fp32 [nG, M] when a_scale varies with g, else NULL
    const float *row_scale;     // fp32 [M] applied at the end, or NULL
    void *C;
    long ldc;
    int *err;
};

RKB_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
          "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
          "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]),
          "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
          "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
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
// (1024 + u) - bias as an fp16 pair: exact for the code ranges used here
RKB_DEV uint32_t h2_sub(uint32_t x, uint32_t bias) {
    __half2 hx = *reinterpret_cast<__half2 *>(&x);
    __half2 hb = *reinterpret_cast<__half2 *>(&bias);
    __half2 r = __hsub2(hx, hb);
    return *reinterpret_cast<uint32_t *>(&r);
}
// 8 offset-by-8 int4 codes (even k in the low nibble) -> 4 fp16 pairs of the
// signed values, pair j = codes 2j, 2j+1
RKB_DEV void widen8_i4(uint32_t u, uint32_t *o) {
    const uint32_t e = u & 0x0F0F0F0Fu, od = (u >> 4) & 0x0F0F0F0Fu;
    o[0] = h2_sub(lop_and_or(prmt(e, od, 0x4400u), 0x00FF00FFu, 0x64006400u), 0x64086408u);
    o[1] = h2_sub(lop_and_or(prmt(e, od, 0x5511u), 0x00FF00FFu, 0x64006400u), 0x64086408u);
    o[2] = h2_sub(lop_and_or(prmt(e, od, 0x6622u), 0x00FF00FFu, 0x64006400u), 0x64086408u);
    o[3] = h2_sub(lop_and_or(prmt(e, od, 0x7733u), 0x00FF00FFu, 0x64006400u), 0x64086408u);
}
// 4 offset-by-128 int8 codes -> 2 fp16 pairs of the signed values
RKB_DEV void widen4_i8(uint32_t w, uint32_t *o) {
    o[0] = h2_sub(prmt(w, 0x64646464u, 0x5140u), 0x64806480u);
    o[1] = h2_sub(prmt(w, 0x64646464u, 0x7362u), 0x64806480u);
}

template <int WBITS, int OUT, bool AS_COL>
__global__ void __launch_bounds__(NUM_THREADS, 1)
wgemm_xp_kernel(const __grid_constant__ CUtensorMap tmB, const Args g) {
    using C = Cfg<WBITS>;
    constexpr int RS = C::RS;
    constexpr int RB = 64 * WBITS / 8;               // code bytes per row of a 64-wide K block
    constexpr uint32_t IDESC = idesc_f16_f32acc(WM, NT);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + RS * C::RAW_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBARS);
    const uint32_t sbase = smem_u32(smem);
    auto sB = [&](int r) { return sbase + r * C::RAW_BYTES; };
    auto sCode = [&](int r) { return sbase + r * C::RAW_BYTES + C::B_BYTES; };
    auto pCode = [&](int r) { return smem + r * C::RAW_BYTES + C::B_BYTES; };
    auto raw_full = [&](int r) { return smem_u32(&bars[r]); };
    auto raw_empty = [&](int r) { return smem_u32(&bars[RS + r]); };
    auto a_full = [&](int a) { return smem_u32(&bars[2 * RS + a]); };
    auto a_empty = [&](int a) { return smem_u32(&bars[2 * RS + DA + a]); };
    auto p_full = [&](int b) { return smem_u32(&bars[2 * RS + 2 * DA + b]); };
    auto p_empty = [&](int b) { return smem_u32(&bars[2 * RS + 2 * DA + 2 + b]); };
    const uint32_t drain_bar = smem_u32(&bars[2 * RS + 2 * DA + 4]);
    auto acol = [&](int a) { return A_COL0 + static_cast<uint32_t>(a * ACOLS); };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmB);
        for (int r = 0; r < RS; ++r) {
            mbar_init(raw_full(r), 1);
            mbar_init(raw_empty(r), 1);
        }
        for (int a = 0; a < DA; ++a) {
            mbar_init(a_full(a), NUM_DEQ);
            mbar_init(a_empty(a), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(p_full(b), 1);
            mbar_init(p_empty(b), NUM_EPI);
        }
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
    const int seg_steps = g.seg / 16;            // MMA K-steps per segment
    const int k_steps = g.K / 16;                // K % 32 == 0: the padded tail is never issued
    const int nseg = g.K / g.seg;

    if (warp == 0) {
        if (lane == 0) {
            int r = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int mt = t % g.m_tiles, nt128 = t / g.m_tiles;
                // half h of 256-row tile t256 in the ragged layout (rkb_wlayout.cuh):
                // rows past the weight's end are not stored and keep stale data
                const int t256 = nt128 >> 1, h = nt128 & 1;
                const int rows = wl_rows(g.N, t256);
                const int hv = rows - h * WM < WM ? rows - h * WM : WM;
                const uint32_t cbytes = static_cast<uint32_t>(hv * RB);
                for (int kb = 0; kb < g.k_blocks; ++kb) {
                    if (!mbar_wait(raw_empty(r), ph ^ 1, g.err, ERR_WAIT_PRODUCER)) { ok = false; break; }
                    mbar_arrive_expect_tx(raw_full(r), NT * 128 + cbytes);
                    tma_load_2d(sB(r), &tmB, kb * 64, mt * NT, raw_full(r));
                    bulk_load(sCode(r), g.codes + wl_block(g.N, g.kb64_total, t256, kb, RB) + h * WM * RB,
                              cbytes, raw_full(r));
                    if (++r == RS) { r = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int r = 0, a = 0;
            uint32_t aph = 0;
            uint32_t s = 0;            // segments issued by this CTA (P buffer s & 1)
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                for (int kb = 0; kb < g.k_blocks && ok; ++kb) {
                    // a_full(a) implies raw_full(r): the dequantisers waited for it
                    if (!mbar_wait(a_full(a), aph, g.err, ERR_WAIT_MMA_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t bdesc = smem_desc_sw128(sB(r));
#pragma unroll 1
                    for (int k = 0; k < 4; ++k) {
                        const int ks = kb * 4 + k;
                        if (ks >= k_steps) break;
                        const int pos = ks % seg_steps;
                        const uint32_t b = s & 1;
                        if (pos == 0) {
                            if (!mbar_wait(p_empty(b), ((s >> 1) & 1) ^ 1, g.err, ERR_WAIT_MMA_ACC)) { ok = false; break; }
                            tc_fence_after();
                        }
                        tc_mma_f16_ts(tmem_base + b * NT, tmem_base + acol(a) + k * 8,
                                      bdesc + static_cast<uint64_t>(k * 2), IDESC, pos != 0);
                        if (pos == seg_steps - 1) {
                            tc_commit(p_full(b));
                            ++s;
                        }
                    }
                    tc_commit(raw_empty(r));
                    tc_commit(a_empty(a));
                    if (++r == RS) r = 0;
                    if (++a == DA) { a = 0; aph ^= 1; }
                }
            }
            if (!ok) {
                tc_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0);
            }
        }
    } else if (warp < EPI_WARP0) {
        // dequantisers: warp q owns TMEM lanes 32q..32q+31 = weight rows
        const int q = warp & 3;
        const int row = q * 32 + lane;
        int r = 0, a = 0;
        uint32_t rph = 0, aph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < g.k_blocks; ++kb) {
                if (!mbar_wait_warp(raw_full(r), rph, g.err, ERR_WAIT_DEQUANT) ||
                    !mbar_wait_warp(a_empty(a), aph ^ 1, g.err, ERR_WAIT_DEQUANT)) { ok = false; break; }
                uint32_t o[32];
                if (WBITS == 4) {
                    const uint4 u0 = *reinterpret_cast<const uint4 *>(pCode(r) + row * 32);
                    const uint4 u1 = *reinterpret_cast<const uint4 *>(pCode(r) + row * 32 + 16);
                    widen8_i4(u0.x, o + 0);  widen8_i4(u0.y, o + 4);
                    widen8_i4(u0.z, o + 8);  widen8_i4(u0.w, o + 12);
                    widen8_i4(u1.x, o + 16); widen8_i4(u1.y, o + 20);
                    widen8_i4(u1.z, o + 24); widen8_i4(u1.w, o + 28);
                } else {
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const uint4 u = *reinterpret_cast<const uint4 *>(pCode(r) + row * 64 + v * 16);
                        widen4_i8(u.x, o + 8 * v + 0);
                        widen4_i8(u.y, o + 8 * v + 2);
                        widen4_i8(u.z, o + 8 * v + 4);
                        widen4_i8(u.w, o + 8 * v + 6);
                    }
                }
                tmem_st32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acol(a), o);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full(a));
                if (++r == RS) { r = 0; rph ^= 1; }
                if (++a == DA) { a = 0; aph ^= 1; }
            }
        }
    } else {
        // epilogue: lane = weight row n; token columns 32j..32j+31 of the tile
        const int e = warp - EPI_WARP0;
        const int q = warp & 3, j = e >> 2;
        const uint32_t tl = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + j * 32;
        uint32_t s = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            const int mt = t % g.m_tiles, nt128 = t / g.m_tiles;
            const int n = nt128 * WM + q * 32 + lane;
            const int m0 = mt * NT + j * 32;
            const bool n_ok = n < g.N;
            const float *bsrow = g.b_scale + static_cast<size_t>(n_ok ? n : 0) * g.nG;
            float acc[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) acc[c] = 0.f;
            for (int si = 0; si < nseg; ++si, ++s) {
                const int grp = si * g.seg / g.group;
                const float bs = n_ok ? __ldg(bsrow + grp) : 0.f;
                float as_l = 0.f;
                if (AS_COL) as_l = (m0 + lane < g.M) ? __ldg(g.a_scale_t + static_cast<size_t>(grp) * g.M + m0 + lane) : 0.f;
                const uint32_t b = s & 1;
                if (!mbar_wait_warp(p_full(b), (s >> 1) & 1, g.err, ERR_WAIT_EPILOGUE)) { ok = false; break; }
                tc_fence_after();
                uint32_t v[32];
                tmem_ld32(tl + b * NT, v);
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_empty(b));
                if (AS_COL) {
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        acc[c] = fmaf(bs * __shfl_sync(0xffffffffu, as_l, c), __uint_as_float(v[c]), acc[c]);
                } else {
                    const float2 bs2 = make_float2(bs, bs);
#pragma unroll
                    for (int c = 0; c < 32; c += 2) {
                        float2 x = __ffma2_rn(bs2, make_float2(__uint_as_float(v[c]), __uint_as_float(v[c + 1])),
                                              make_float2(acc[c], acc[c + 1]));
                        acc[c] = x.x;
                        acc[c + 1] = x.y;
                    }
                }
            }
            if (!ok) break;
            // the chunk's 32 token scales: lane c loads token m0 + c, then broadcast
            const float rs_l = (g.row_scale && m0 + lane < g.M) ? __ldg(g.row_scale + m0 + lane) : 1.0f;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const float x = acc[c] * __shfl_sync(0xffffffffu, rs_l, c);
                const int m = m0 + c;
                if (m < g.M && n_ok) {
                    const long off = static_cast<long>(m) * g.ldc + n;
                    if (OUT == RKB_OUT_F32) static_cast<float *>(g.C)[off] = x;
                    else static_cast<__half *>(g.C)[off] = __float2half_rn(x);
                }
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

template <int WBITS, int OUT, bool AS_COL>
int launch(const rkb_wgemm_desc *d, int *err, cudaStream_t stream) {
    using C = Cfg<WBITS>;
    static std::once_flag attr_once[16];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 15], [] {
        cudaFuncSetAttribute(wgemm_xp_kernel<WBITS, OUT, AS_COL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM);
    });
    const int sms = rkb_device_sm_count(dev);
    Args g;
    g.M = d->M; g.N = d->N; g.K = d->K;
    g.n_tiles = (d->N + WM - 1) / WM;
    g.m_tiles = (d->M + NT - 1) / NT;
    CUtensorMap tb;
    if (make_tmap_2d(&tb, d->A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, d->K, d->M, d->lda, 64, NT))
        return ROCKET_E_SHAPE;
    const int kp = (d->K + 127) / 128 * 128;
    g.kb64_total = kp / 64;
    g.k_blocks = (d->K + 63) / 64;
    g.group = d->group;
    g.seg = d->seg;
    g.nG = d->K / d->group;
    g.codes = static_cast<const uint8_t *>(d->Wq);
    g.b_scale = d->b_scale;
    g.a_scale_t = d->a_scale_t;
    g.row_scale = d->row_scale;
    g.C = d->C; g.ldc = d->ldc;
    g.err = err;
    const int tiles = g.m_tiles * g.n_tiles;
    const int grid = tiles < sms ? tiles : sms;
    wgemm_xp_kernel<WBITS, OUT, AS_COL><<<grid, NUM_THREADS, C::SMEM, stream>>>(tb, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "rkb wgemm_xp launch: %s\n", cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    return 0;
}

}  // namespace wxp
}  // namespace rkb

// Segment length for exact partials: the whole group, or for int8 weights a
// group wider than 1024 cut into equal pieces of at most 1024 (|a w| <= 2^14,
// so a piece's sum stays within fp32's exact integer range 2^24).
extern "C" int rkb_wgemm_xp_segment(int group, int w_bits) {
    if (group <= 0 || group % 32) return ROCKET_E_SHAPE;
    const int cap = w_bits == 4 ? 16384 : 1024;
    if (group <= cap) return group;
    for (int s = cap / 32 * 32; s >= 32; s -= 32)
        if (group % s == 0) return s;
    return 32;
}

extern "C" int rkb_wgemm_xp_run(const rkb_wgemm_desc *d, int *err, cudaStream_t stream) {
    using namespace rkb::wxp;
    if (d->M <= 0 || d->N <= 0 || d->K <= 0 || d->K % 32 || !d->a_f16 || !d->b_scale ||
        d->group <= 0 || d->K % d->group || d->seg <= 0 || d->seg % 32 || d->group % d->seg ||
        (d->lda * 2) % 16)
        return ROCKET_E_SHAPE;
#define RKB_XP(BITS, OUT)                                                        \
    return d->a_scale_t ? launch<BITS, OUT, true>(d, err, stream)                \
                        : launch<BITS, OUT, false>(d, err, stream)
    if (d->w_bits == 4) {
        if (d->out_kind == RKB_OUT_F32) { RKB_XP(4, RKB_OUT_F32); }
        if (d->out_kind == RKB_OUT_F16) { RKB_XP(4, RKB_OUT_F16); }
    } else if (d->w_bits == 8) {
        if (d->out_kind == RKB_OUT_F32) { RKB_XP(8, RKB_OUT_F32); }
        if (d->out_kind == RKB_OUT_F16) { RKB_XP(8, RKB_OUT_F16); }
    }
#undef RKB_XP
    return ROCKET_E_UNSUPPORTED;
}
