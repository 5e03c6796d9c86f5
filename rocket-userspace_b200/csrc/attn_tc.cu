// attn_tc.cu -- fused multi-head self-attention core on the sm_100a tensor
// cores: O = softmax(Q K^T * scale) V per (batch, head), never writing the
// T x T score matrix to HBM.
//
// Replaces the attention inner loop of the reference's rocket_mha_self_fp16
// (src/rocket_attn.c:92-176: per head a scores matmul, key padding to %32 with
// -30000 masking, a composed NPU softmax, and a P.V matmul), whose definition
// is the fp64 host loop at src/rocket_attn.c:41-84.
//
// One CTA = 128 queries of one (batch, head); head_dim 64.  Roles:
//   warp 0      TMA: Q once; K blocks of 128 keys into a 2-deep ring, V^T
//               blocks into one buffer (two CTAs fit on an SM)
//   warp 1      MMA issuer: S_j = Q K_j^T (M=128, N=128, fp32 in TMEM cols
//               0..127), O_j = P_j V_j (M=128, N=64, TMEM cols 128..191); S_{j+1}
//               is issued as soon as S_j has been read, so it overlaps the
//               softmax of block j
//   warps 2..9  softmax, two warps per TMEM lane quarter: each thread owns one
//               query row and half of every 128-key block; it reads its 64
//               scores from TMEM twice, 32 at a time (row max, then weights),
//               exchanges half-block row maxima with its partner through
//               shared memory (an mbarrier with a bounded wait), computes exp2
//               weights and its part of the row sum in fp32, rescales its 32
//               columns of O in TMEM when the row's reference max moved by
//               more than 2^8, and writes its 64-key panel of P_j as fp16
//               into the 128-byte-swizzled shared tile for the P V MMA; the
//               two partial row sums are added at the end
// About 100 KB of shared memory, 256 TMEM columns and 85 registers a thread,
// so two CTAs share an SM.
// Keys past T (the last block) are masked to -inf.  Inputs come from
// rkb_split_heads: Q, K [B*H, Tp, 64] and V^T [B*H, 64, Tp], zero-padded.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>

#define RKB_SPIN_TRIES 4096   // per-block hand-offs: see rkb_ptx.cuh
#include "rkb_ptx.cuh"
#include "rkb_tmap.h"
#include "../src/rkb_kernels.h"
#include "../../include/rocket_npu.h"

namespace rkb {
namespace attn {

constexpr int BQ = 128, BKV = 128, DH = 64;
constexpr int NUM_THREADS = 320;       // producer, MMA, 8 softmax warps
constexpr int Q_BYTES = BQ * DH * 2;        // 16 KB
constexpr int K_BYTES = BKV * DH * 2;       // 16 KB
constexpr int VT_BYTES = DH * BKV * 2;      // 16 KB (two 64-key panels of 8 KB)
constexpr int P_BYTES = BQ * BKV * 2;       // 32 KB (two 64-key panels of 16 KB)
// Shared memory fits two CTAs per SM (~98 KB each): K in a 2-deep ring (K_{j+1}
// is needed as soon as S_j has been read), V^T and P single-buffered (V_j is
// read only by P_j V_j, which runs a whole softmax step after S_j).
constexpr int K_STAGES = 2;
constexpr int OFF_Q = 0;
constexpr int OFF_K = Q_BYTES;
constexpr int OFF_V = OFF_K + K_STAGES * K_BYTES;
constexpr int OFF_P = OFF_V + VT_BYTES;
constexpr int OFF_X = OFF_P + P_BYTES;        // row-max exchange [2 parities][2 halves][128]; the
constexpr int X_BYTES = 2 * 2 * BQ * 4;       // final row sums reuse the parity not read last
constexpr int OFF_BAR = OFF_X + X_BYTES;
constexpr int NBARS = 1 + 2 * K_STAGES + 2 + 5 + 8;
constexpr float RESCALE_LOG2 = 8.f;    // the reference max moves only when a row's max grows by > 2^8
constexpr int SMEM = OFF_BAR + NBARS * 8 + 16 + 1024;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t S_COL = 0, O_COL = 128;

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

struct Args {
    int T, Tp, H, nkb;
    float scale_log2;     // softmax scale * log2(e)
    __half *out;
    long ldo;
    int *err;
};

__global__ void __launch_bounds__(NUM_THREADS, 2)
attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmVt, const Args g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t sb = smem_u32(smem);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBARS);
    const uint32_t q_full = smem_u32(&bars[0]);
    auto k_full = [&](int s) { return smem_u32(&bars[1 + s]); };
    auto k_empty = [&](int s) { return smem_u32(&bars[1 + K_STAGES + s]); };
    const uint32_t v_full = smem_u32(&bars[1 + 2 * K_STAGES]);
    const uint32_t v_empty = smem_u32(&bars[2 + 2 * K_STAGES]);
    constexpr int KV_STAGES = K_STAGES + 1;   // offsets of the barriers below
    const uint32_t s_full = smem_u32(&bars[1 + 2 * KV_STAGES]);
    const uint32_t s_free = smem_u32(&bars[2 + 2 * KV_STAGES]);
    const uint32_t p_full = smem_u32(&bars[3 + 2 * KV_STAGES]);
    // P_j V_j done (it read P buffer j & 1 and accumulated into O): completion k
    // of pv_done(b) is block b + 2k, so block j waits parity (j >> 1) & 1
    auto pv_done = [&](int b) { return smem_u32(&bars[4 + 2 * KV_STAGES + b]); };
    // per TMEM lane quarter: the two softmax warps of those rows exchange their
    // half-block row maxima (every block) and their row sums (at the end)
    auto xmax_bar = [&](int q) { return smem_u32(&bars[6 + 2 * KV_STAGES + q]); };
    auto xsum_bar = [&](int q) { return smem_u32(&bars[10 + 2 * KV_STAGES + q]); };
    auto sK = [&](int s) { return sb + OFF_K + s * K_BYTES; };
    const uint32_t sVt = sb + OFF_V;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x, bh = blockIdx.y;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmVt);
        mbar_init(q_full, 1);
        for (int s = 0; s < K_STAGES; ++s) {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
        }
        mbar_init(v_full, 1);
        mbar_init(v_empty, 1);
        mbar_init(s_full, 1);
        mbar_init(s_free, 8);
        mbar_init(p_full, 8);
        mbar_init(pv_done(0), 1);
        mbar_init(pv_done(1), 1);
        for (int q = 0; q < 4; ++q) {
            mbar_init(xmax_bar(q), 64);
            mbar_init(xsum_bar(q), 64);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nkb = g.nkb;

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, Q_BYTES);
            tma_load_2d(sb + OFF_Q, &tmQ, 0, bh * g.Tp + qt * BQ, q_full);
            // order: K_0, then K_{j+1} ahead of V_j (V_j waits for P_{j-1} V_{j-1})
            auto load_k = [&](int j) {
                const int s = j % K_STAGES;
                if (!mbar_wait(k_empty(s), ((j / K_STAGES) & 1) ^ 1, g.err, ERR_WAIT_PRODUCER)) return false;
                mbar_arrive_expect_tx(k_full(s), K_BYTES);
                tma_load_2d(sK(s), &tmK, 0, bh * g.Tp + j * BKV, k_full(s));
                return true;
            };
            bool ok = nkb > 0 && load_k(0);
            for (int j = 0; j < nkb && ok; ++j) {
                if (j + 1 < nkb && !load_k(j + 1)) break;
                if (!mbar_wait(v_empty, (j & 1) ^ 1, g.err, ERR_WAIT_PRODUCER)) break;
                mbar_arrive_expect_tx(v_full, VT_BYTES);
                tma_load_2d(sVt, &tmVt, j * BKV, bh * DH, v_full);
                tma_load_2d(sVt + VT_BYTES / 2, &tmVt, j * BKV + 64, bh * DH, v_full);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDS = idesc_f16_f32acc(BQ, BKV);
            constexpr uint32_t IDO = idesc_f16_f32acc(BQ, DH);
            bool ok = mbar_wait(q_full, 0, g.err, ERR_WAIT_MMA_FULL) &&
                      mbar_wait(k_full(0), 0, g.err, ERR_WAIT_MMA_FULL);
            if (ok) {
                tc_fence_after();
                const uint64_t qd = smem_desc_sw128(sb + OFF_Q), kd = smem_desc_sw128(sK(0));
#pragma unroll
                for (int k = 0; k < 4; ++k) tc_mma_f16(tmem + S_COL, qd + 2 * k, kd + 2 * k, IDS, k > 0);
                tc_commit(s_full);
                tc_commit(k_empty(0));
            }
            for (int j = 0; j < nkb && ok; ++j) {
                if (j + 1 < nkb) {
                    const int s1 = (j + 1) % K_STAGES;
                    if (!mbar_wait(k_full(s1), ((j + 1) / K_STAGES) & 1, g.err, ERR_WAIT_MMA_FULL) ||
                        !mbar_wait(s_free, j & 1, g.err, ERR_WAIT_MMA_ACC)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t qd = smem_desc_sw128(sb + OFF_Q), kd = smem_desc_sw128(sK(s1));
#pragma unroll
                    for (int k = 0; k < 4; ++k) tc_mma_f16(tmem + S_COL, qd + 2 * k, kd + 2 * k, IDS, k > 0);
                    tc_commit(s_full);
                    tc_commit(k_empty(s1));
                }
                if (!mbar_wait(p_full, j & 1, g.err, ERR_WAIT_MMA_FULL) ||
                    !mbar_wait(v_full, j & 1, g.err, ERR_WAIT_MMA_FULL)) { ok = false; break; }
                tc_fence_after();
                const uint32_t pbuf = sb + OFF_P;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t pd = smem_desc_sw128(pbuf + (kk >> 2) * (P_BYTES / 2) + (kk & 3) * 32);
                    const uint64_t vd = smem_desc_sw128(sVt + (kk >> 2) * (VT_BYTES / 2) + (kk & 3) * 32);
                    tc_mma_f16(tmem + O_COL, pd, vd, IDO, (j | kk) != 0);   // O accumulates in TMEM
                }
                tc_commit(pv_done(j & 1));
                tc_commit(v_empty);
            }
            if (!ok) {
                tc_commit(q_full);   // drain: arrives once every issued MMA has finished
                mbar_wait_drain(q_full, 1);
            }
        }
    } else {
        // softmax: warps 2..9; warp pair (e, e + 4) shares TMEM lane quarter q
        // (query rows 32q..32q+31) and takes key half `half` of every block
        const int e = warp - 2;
        const int q4 = warp & 3;
        const int half = e >> 2;
        const int row = q4 * 32 + lane;
        const uint32_t tl = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
        float *xm = reinterpret_cast<float *>(smem + OFF_X);        // [parity][half][row]
        constexpr int HK = BKV / 2;                                 // keys per warp per block
        constexpr int HD = DH / 2;                                  // output columns per warp
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkb; ++j) {
            if (!mbar_wait_warp(s_full, j & 1, g.err, ERR_WAIT_EPILOGUE)) { ok = false; break; }
            tc_fence_after();
            // the scores stay in TMEM and are read twice, 32 at a time (max, then
            // weights), which keeps the thread within the register budget of
            // two CTAs per SM.  The scale (> 0) is folded into the exponent:
            // max over raw scores, weights ex2(s * scale_log2 - m); keys past T
            // exist only in the last block.
            const int kbase = j * BKV + half * HK;
            const bool tail = j * BKV + BKV > g.T;
            float mr = -INFINITY;
#pragma unroll
            for (int c = 0; c < HK; c += 32) {
                uint32_t r[32];
                tmem_ld32(tl + S_COL + half * HK + c, r);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (!tail || kbase + c + i < g.T) mr = fmaxf(mr, __uint_as_float(r[i]));
            }
            // exchange half-block maxima with the partner warp (bounded wait)
            xm[((j & 1) * 2 + half) * BQ + row] = mr;
            mbar_arrive(xmax_bar(q4));
            if (!mbar_wait_warp(xmax_bar(q4), j & 1, g.err, ERR_WAIT_EPILOGUE)) { ok = false; break; }
            mr = fmaxf(mr, xm[((j & 1) * 2 + (half ^ 1)) * BQ + row]) * g.scale_log2;
            // lazy rescale: keep the reference max unless this block exceeds it by 2^8
            const float m_new = mr > m + RESCALE_LOG2 ? mr : m;
            const float alpha = m_new == m ? 1.f : ex2_approx(m - m_new);   // 0 on the first block
            // P_{j-1} V_{j-1} has read the single P buffer and written O
            if (j > 0 && !mbar_wait_warp(pv_done((j - 1) & 1), ((j - 1) >> 1) & 1, g.err, ERR_WAIT_EPILOGUE)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // O (in TMEM) holds P_0..P_{j-1} V: rescale this warp's 32 columns in
            // place when a row's reference max moved (both warps of the pair see
            // the same rows, so they decide alike)
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                uint32_t r[32];
                tmem_ld32(tl + O_COL + half * HD, r);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                tmem_st32(tl + O_COL + half * HD, r);
                tmem_st_wait();
            }
            // P_j as fp16: this warp's 64 keys are panel `half` of the swizzled A tile
            uint8_t *prow = smem + OFF_P + half * (P_BYTES / 2) + row * 128;
            float sum = 0.f;
#pragma unroll
            for (int cc = 0; cc < HK; cc += 32) {
                uint32_t r[32];
                tmem_ld32(tl + S_COL + half * HK + cc, r);
                tmem_ld_wait();
                float pv[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float sv = (!tail || kbase + cc + i < g.T) ? __uint_as_float(r[i]) : -INFINITY;
                    pv[i] = ex2_approx(fmaf(sv, g.scale_log2, -m_new));
                    sum += pv[i];
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t hv[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        __half2 p = __floats2half2_rn(pv[c * 8 + 2 * i], pv[c * 8 + 2 * i + 1]);
                        hv[i] = *reinterpret_cast<uint32_t *>(&p);
                    }
                    const int ch = cc / 8 + c;
                    *reinterpret_cast<uint4 *>(prow + ((ch ^ (row & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                }
            }
            l = l * alpha + sum;                      // this warp's half of the row sum
            m = m_new;
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(s_free);                  // S_j fully read: S_{j+1} may overwrite it
                mbar_arrive(p_full);
            }
        }
        if (ok && nkb > 0 &&
            mbar_wait_warp(pv_done((nkb - 1) & 1), ((nkb - 1) >> 1) & 1, g.err, ERR_WAIT_EPILOGUE)) {
            tc_fence_after();
            uint32_t r[32];
            tmem_ld32(tl + O_COL + half * HD, r);
            tmem_ld_wait();
            // the row sum is the two halves' sum (a + b == b + a: both warps agree);
            // exchanged through the max-exchange slots of the parity not read last
            float *xs = xm + (nkb & 1) * 2 * BQ;          // [half][row]
            xs[half * BQ + row] = l;
            mbar_arrive(xsum_bar(q4));
            if (mbar_wait_warp(xsum_bar(q4), 0, g.err, ERR_WAIT_EPILOGUE)) {
                const float lt = l + xs[(half ^ 1) * BQ + row];
                const int t = qt * BQ + row;
                if (t < g.T) {
                    const int b = bh / g.H, h = bh % g.H;
                    __half *dst = g.out + static_cast<long>(b * g.T + t) * g.ldo + h * DH + half * HD;
                    const float inv = 1.f / lt;
#pragma unroll
                    for (int c = 0; c < HD; c += 8) {
                        uint32_t w[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            __half2 p = __floats2half2_rn(__uint_as_float(r[c + 2 * i]) * inv,
                                                          __uint_as_float(r[c + 2 * i + 1]) * inv);
                            w[i] = *reinterpret_cast<uint32_t *>(&p);
                        }
                        *reinterpret_cast<uint4 *>(dst + c) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
        tc_fence_before();
    }

    __syncwarp();   // reconverge role-divergent lanes: the barrier below is warp-aligned
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace attn
}  // namespace rkb

extern "C" int rkb_attention(const void *Q, const void *K, const void *Vt, int B, int H, int T, int Tp,
                             int dh, float scale, void *out, long ldo, int *err, cudaStream_t stream) {
    using namespace rkb::attn;
    if (dh != DH || Tp % BKV || T > Tp || T <= 0 || (ldo % 8)) return ROCKET_E_UNSUPPORTED;
    static std::once_flag once[16];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 15], [] {
        cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        cudaFuncSetAttribute(attn_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    });
    CUtensorMap tq, tk, tv;
    const long BH = static_cast<long>(B) * H;
    if (rkb::make_tmap_2d(&tq, Q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, DH, BH * Tp, DH, 64, BQ) ||
        rkb::make_tmap_2d(&tk, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, DH, BH * Tp, DH, 64, BKV) ||
        rkb::make_tmap_2d(&tv, Vt, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Tp, BH * DH, Tp, 64, DH))
        return ROCKET_E_SHAPE;
    Args g;
    g.T = T; g.Tp = Tp; g.H = H; g.nkb = Tp / BKV;
    g.scale_log2 = scale * 1.4426950408889634f;
    g.out = static_cast<__half *>(out);
    g.ldo = ldo;
    g.err = err;
    dim3 grid(Tp / BQ, static_cast<unsigned>(BH));
    attn_kernel<<<grid, NUM_THREADS, SMEM, stream>>>(tq, tk, tv, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "rkb attention launch: %s\n", cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    return 0;
}
