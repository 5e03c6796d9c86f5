// fa_tc.cu -- masked grouped-query flash attention on the sm_100a tensor cores:
// per query head h (kv head hk = h / (n_head / n_kv_heads)),
//   S = scale * q_h k_hk^T  [softcap: S = softcap * tanh(S / softcap)]
//   S = max(S + mask, -30000);  P = softmax(S);  out_h = P v_hk
// without writing the score matrix anywhere.
//
// Replaces the reference's rocket_flash_attn_fp16 / _mt / _ctx
// (src/rocket_attn.c:700-900: per-head QK matmul, host-side mask + softmax,
// AV matmul), whose definition is the host loop at src/rocket_attn.c:181-222
// (fa_score: scale, soft-cap, additive mask, clamp at -30000).
//
// Layouts (the reference's, head-major):
//   Q [n_head][T][dh]   K [n_kv_heads][n_kv][dh]   V [n_kv_heads][dv][n_kv]
//   mask [T][n_kv] additive fp16 (optional)        out [n_head][T][dv]
// V's [dv][n_kv] rows are already the K-major B operand of O = P V.
//
// One CTA = 128 queries of one head.  head_dim is loaded as 64-wide panels
// (1..4; TMA zero-fills columns past dh), keys in blocks of BKV (128 when
// dh <= 128 and dv <= 128, else 64 so two K/V stages fit in shared memory).
//   warp 0      TMA: Q once; K (dh panels) and V (64-key panels) per block
//               into a 2-stage ring
//   warp 1      MMA: S_j = Q K_j^T into TMEM; S_{j+1} as soon as S_j is read;
//               O += P_j V_j into a TMEM accumulator of dv columns
//   warps 2..5  one query row per thread: scores from TMEM, the reference's
//               score transform, online softmax in the log2 domain with lazy
//               rescaling (the running max moves only when a row's max grows
//               by more than 2^8; O in TMEM is then rescaled with
//               tcgen05.ld / st), P_j as fp16 into a swizzled shared tile
// Keys past n_kv score -inf (they do not exist in the reference); masked keys
// clamp to -30000 like the reference, so a fully masked row averages V.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>

#include "rkb_ptx.cuh"
#include "rkb_tmap.h"
#include "../src/rkb_kernels.h"
#include "../../include/rocket_npu.h"

namespace rkb {
namespace fa {

constexpr int BQ = 128;
constexpr int NUM_THREADS = 192;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_LOG2 = 8.f;     // P values stay below 2^8 between rescales

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
    int T, n_kv, dv, n_head, gqa, dhp, nkb;
    int q_rows, kv_rows;   // rows per head in the Q / K tensor maps (>= T / n_kv)
    int hb;                // heads per output batch: out(h, t) = out + (h / hb) * bstride + (h % hb) * dv + t * ldo
    long bstride, ldo;
    float scale, softcap;
    const __half *mask;
    int mask_vec;          // mask rows 16-byte aligned (n_kv % 8 == 0, aligned base)
    __half *out;
    int *err;
};

// Shared-memory plan (offsets from a 1024-aligned base)
struct Plan {
    int q, kv, k_bytes, v_bytes, stage, p, bar, total;
};
__host__ __device__ inline Plan plan_for(int bkv, int dhp, int dv) {
    Plan p;
    p.q = 0;
    p.k_bytes = dhp * bkv * 128;
    p.v_bytes = (bkv / 64) * dv * 128;
    p.stage = p.k_bytes + p.v_bytes;
    p.kv = dhp * BQ * 128;
    p.p = p.kv + 2 * p.stage;
    p.bar = p.p + (bkv / 64) * BQ * 128;
    p.total = p.bar + 16 * 8 + 16 + 1024;
    return p;
}

// MASK: 0 none, 1 16-byte vector loads, 2 scalar loads; CAP: soft-cap on.
// Separate instantiations keep the fully unrolled score loop free of the
// branches (and the tanh code) a call does not use.
template <int BKV, int MASK, bool CAP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
fa_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
          const __grid_constant__ CUtensorMap tmV, const Args g) {
    constexpr int KV_STAGES = 2;
    constexpr uint32_t S_COL = 0;
    constexpr uint32_t O_COL = BKV == 128 ? 128 : 256;
    constexpr uint32_t TMEM_COLS = BKV == 128 ? 256 : 512;
    constexpr int NPAN = BKV / 64;      // 64-key panels per block

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t sb = smem_u32(smem);
    const Plan pl = plan_for(BKV, g.dhp, g.dv);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + pl.bar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 16);
    const uint32_t q_full = smem_u32(&bars[0]);
    auto kv_full = [&](int s) { return smem_u32(&bars[1 + s]); };
    auto kv_empty = [&](int s) { return smem_u32(&bars[3 + s]); };
    const uint32_t s_full = smem_u32(&bars[5]);
    const uint32_t s_free = smem_u32(&bars[6]);
    const uint32_t p_full = smem_u32(&bars[7]);
    const uint32_t o_full = smem_u32(&bars[8]);
    auto sK = [&](int s) { return sb + pl.kv + s * pl.stage; };
    auto sV = [&](int s) { return sb + pl.kv + s * pl.stage + pl.k_bytes; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x, h = blockIdx.y;
    const int hk = h / g.gqa;
    const int nkb = g.nkb, dhp = g.dhp, dv = g.dv;

    if (threadIdx.x == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        mbar_init(q_full, 1);
        for (int s = 0; s < KV_STAGES; ++s) {
            mbar_init(kv_full(s), 1);
            mbar_init(kv_empty(s), 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        mbar_init(p_full, 4);
        mbar_init(o_full, 1);
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

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, dhp * BQ * 128);
            for (int p = 0; p < dhp; ++p)
                tma_load_2d(sb + pl.q + p * BQ * 128, &tmQ, p * 64, h * g.q_rows + qt * BQ, q_full);
            for (int j = 0; j < nkb; ++j) {
                const int s = j % KV_STAGES;
                const uint32_t ph = (j / KV_STAGES) & 1;
                if (!mbar_wait(kv_empty(s), ph ^ 1, g.err, ERR_WAIT_PRODUCER)) break;
                mbar_arrive_expect_tx(kv_full(s), pl.stage);
                for (int p = 0; p < dhp; ++p)
                    tma_load_2d(sK(s) + p * BKV * 128, &tmK, p * 64, hk * g.kv_rows + j * BKV, kv_full(s));
                for (int c = 0; c < NPAN; ++c)
                    tma_load_2d(sV(s) + c * dv * 128, &tmV, j * BKV + c * 64, hk * dv, kv_full(s));
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDS = idesc_f16_f32acc(BQ, BKV);
            const uint32_t IDO = idesc_f16_f32acc(BQ, dv);
            auto issue_s = [&](int s) {
                for (int p = 0; p < dhp; ++p) {
                    const uint64_t qd = smem_desc_sw128(sb + pl.q + p * BQ * 128);
                    const uint64_t kd = smem_desc_sw128(sK(s) + p * BKV * 128);
#pragma unroll
                    for (int k = 0; k < 4; ++k) tc_mma_f16(tmem + S_COL, qd + 2 * k, kd + 2 * k, IDS, (p | k) != 0);
                }
                tc_commit(s_full);
            };
            bool ok = mbar_wait(q_full, 0, g.err, ERR_WAIT_MMA_FULL) &&
                      mbar_wait(kv_full(0), 0, g.err, ERR_WAIT_MMA_FULL);
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; j < nkb && ok; ++j) {
                if (j + 1 < nkb) {
                    const int s1 = (j + 1) % KV_STAGES;
                    if (!mbar_wait(kv_full(s1), ((j + 1) / KV_STAGES) & 1, g.err, ERR_WAIT_MMA_FULL) ||
                        !mbar_wait(s_free, j & 1, g.err, ERR_WAIT_MMA_ACC)) { ok = false; break; }
                    tc_fence_after();
                    issue_s(s1);
                }
                if (!mbar_wait(p_full, j & 1, g.err, ERR_WAIT_MMA_FULL)) { ok = false; break; }
                tc_fence_after();
                const int s = j % KV_STAGES;
#pragma unroll
                for (int c = 0; c < NPAN; ++c) {
                    const uint64_t pd = smem_desc_sw128(sb + pl.p + c * BQ * 128);
                    const uint64_t vd = smem_desc_sw128(sV(s) + c * dv * 128);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_f16(tmem + O_COL, pd + 2 * kk, vd + 2 * kk, IDO, (j | c | kk) != 0);
                }
                tc_commit(o_full);
                tc_commit(kv_empty(s));
            }
            if (!ok) {
                tc_commit(q_full);   // drain: arrives once every issued MMA has finished
                mbar_wait_drain(q_full, 1);
            }
        }
    } else {
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;
        const int t = qt * BQ + row;
        const uint32_t tl = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
        const float sc2 = g.scale;
        const __half *mrow = (MASK && t < g.T) ? g.mask + static_cast<size_t>(t) * g.n_kv : nullptr;
        float m = -INFINITY, l = 0.f;
        uint8_t *prow = smem + pl.p + row * 128;
        bool ok = true;
        for (int j = 0; j < nkb; ++j) {
            const int kbase = j * BKV;
            // this block's mask values, fetched before the scores arrive
            uint32_t mk[MASK ? BKV / 2 : 1];
            if (MASK) {
                if (mrow) {
                    if (MASK == 1) {
#pragma unroll
                        for (int c = 0; c < BKV; c += 8) {
                            uint4 v = make_uint4(0, 0, 0, 0);
                            if (kbase + c < g.n_kv) v = __ldg(reinterpret_cast<const uint4 *>(mrow + kbase + c));
                            mk[c / 2] = v.x; mk[c / 2 + 1] = v.y; mk[c / 2 + 2] = v.z; mk[c / 2 + 3] = v.w;
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < BKV; c += 2) {
                            const unsigned short lo = kbase + c < g.n_kv ? __ldg(reinterpret_cast<const unsigned short *>(mrow + kbase + c)) : 0;
                            const unsigned short hi = kbase + c + 1 < g.n_kv ? __ldg(reinterpret_cast<const unsigned short *>(mrow + kbase + c + 1)) : 0;
                            mk[c / 2] = lo | (static_cast<uint32_t>(hi) << 16);
                        }
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < BKV / 2; ++c) mk[c] = 0;
                }
            }
            if (!mbar_wait_warp(s_full, j & 1, g.err, ERR_WAIT_EPILOGUE)) { ok = false; break; }
            tc_fence_after();
            float sv[BKV];
#pragma unroll
            for (int c = 0; c < BKV; c += 32) {
                uint32_t r[32];
                tmem_ld32(tl + S_COL + c, r);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[c + i] = __uint_as_float(r[i]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
            // the reference's score (fa_score), then into the log2 domain
            float mx = -INFINITY;
            const int nvalid = g.n_kv - kbase;   // keys of this block that exist
#pragma unroll
            for (int c = 0; c < BKV; ++c) {
                float s = sv[c] * sc2;
                if (CAP) s = g.softcap * tanhf(s / g.softcap);
                if (MASK) {
                    const __half2 mm = *reinterpret_cast<const __half2 *>(&mk[c / 2]);
                    s += (c & 1) ? __high2float(mm) : __low2float(mm);
                }
                s = fmaxf(s, -30000.f);
                s = (c < nvalid) ? s * LOG2E : -INFINITY;
                sv[c] = s;
                mx = fmaxf(mx, s);
            }
            // lazy rescale: keep the reference max unless this block exceeds it by 2^8
            float m_new = m;
            if (mx > m + RESCALE_LOG2) m_new = mx;
            const float alpha = m_new == m ? 1.f : ex2_approx(m - m_new);   // 0 on the first block
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < BKV; ++c) {
                sv[c] = ex2_approx(sv[c] - m_new);
                sum += sv[c];
            }
            l = l * alpha + sum;
            m = m_new;
            // O_{j-1} complete: P is free, and O may be rescaled in place
            if (j > 0) {
                if (!mbar_wait_warp(o_full, (j - 1) & 1, g.err, ERR_WAIT_EPILOGUE)) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
                    for (int c = 0; c < dv; c += 32) {
                        uint32_t r[32];
                        tmem_ld32(tl + O_COL + c, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                        tmem_st32(tl + O_COL + c, r);
                    }
                    tmem_st_wait();
                }
            }
            // P_j as fp16 into the swizzled [128 x BKV] A tile (64-key panels)
#pragma unroll
            for (int cg = 0; cg < BKV / 8; ++cg) {
                uint32_t hv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    __half2 p = __floats2half2_rn(sv[cg * 8 + 2 * i], sv[cg * 8 + 2 * i + 1]);
                    hv[i] = *reinterpret_cast<uint32_t *>(&p);
                }
                const int panel = cg >> 3, c = cg & 7;
                *reinterpret_cast<uint4 *>(prow + panel * BQ * 128 + ((c ^ (row & 7)) << 4)) =
                    make_uint4(hv[0], hv[1], hv[2], hv[3]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok && nkb > 0 && mbar_wait_warp(o_full, (nkb - 1) & 1, g.err, ERR_WAIT_EPILOGUE)) {
            tc_fence_after();
            const float inv = 1.f / l;
            __half *dst = g.out + (h / g.hb) * g.bstride + (h % g.hb) * dv + static_cast<long>(t) * g.ldo;
            for (int c = 0; c < dv; c += 32) {
                uint32_t r[32];
                tmem_ld32(tl + O_COL + c, r);
                tmem_ld_wait();
                if (t < g.T) {
#pragma unroll
                    for (int v8 = 0; v8 < 4; ++v8) {
                        if (c + v8 * 8 < dv) {
                            uint32_t w[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                __half2 p = __floats2half2_rn(__uint_as_float(r[v8 * 8 + 2 * i]) * inv,
                                                              __uint_as_float(r[v8 * 8 + 2 * i + 1]) * inv);
                                w[i] = *reinterpret_cast<uint32_t *>(&p);
                            }
                            *reinterpret_cast<uint4 *>(dst + c + v8 * 8) = make_uint4(w[0], w[1], w[2], w[3]);
                        }
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

template <int BKV, int MASK, bool CAP>
int launch(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv, const Args &g,
           cudaStream_t stream) {
    const Plan pl = plan_for(BKV, g.dhp, g.dv);
    static std::once_flag once[16];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 15], [] {
        cudaFuncSetAttribute(fa_kernel<BKV, MASK, CAP>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    });
    // BKV 64 allocates all 512 TMEM columns: ask for more than half the SM's
    // shared memory so a second CTA never lands on the SM and stalls in alloc
    const int smem = BKV == 64 && pl.total < 116 * 1024 ? 116 * 1024 : pl.total;
    dim3 grid((g.T + BQ - 1) / BQ, static_cast<unsigned>(g.n_head));
    fa_kernel<BKV, MASK, CAP><<<grid, NUM_THREADS, smem, stream>>>(tq, tk, tv, g);
    return 0;
}

template <int BKV>
int launch_kind(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv, const Args &g,
                cudaStream_t stream) {
    const int mask = g.mask ? (g.mask_vec ? 1 : 2) : 0;
    const bool cap = g.softcap != 0.f;
    switch (mask * 2 + (cap ? 1 : 0)) {
    case 0: return launch<BKV, 0, false>(tq, tk, tv, g, stream);
    case 1: return launch<BKV, 0, true>(tq, tk, tv, g, stream);
    case 2: return launch<BKV, 1, false>(tq, tk, tv, g, stream);
    case 3: return launch<BKV, 1, true>(tq, tk, tv, g, stream);
    case 4: return launch<BKV, 2, false>(tq, tk, tv, g, stream);
    default: return launch<BKV, 2, true>(tq, tk, tv, g, stream);
    }
}

}  // namespace fa
}  // namespace rkb

// General form: Q rows of head h start at row h * q_rows of a [n_head * q_rows][dh]
// array, K rows of kv head hk at hk * kv_rows of [n_kv_heads * kv_rows][dh]; V is
// [n_kv_heads * dv] rows of ldv elements; out(h, t) = out + (h / hb) * bstride +
// (h % hb) * dv + t * ldo.  Rows must be 16-byte aligned (dh % 8, ldv % 8, ldo % 8).
// Shapes the kernel does not take return ROCKET_E_UNSUPPORTED: dh > 256,
// dv > 256, dv % 16.
extern "C" int rkb_flash_attn_ex(const void *Q, const void *K, const void *V, long ldv, const void *mask,
                                 void *out, int T, int n_kv, int dh, int dv, int n_head, int n_kv_heads,
                                 float scale, float softcap, int q_rows, int kv_rows, int hb, long bstride,
                                 long ldo, int *err, cudaStream_t stream) {
    using namespace rkb::fa;
    if (T <= 0 || n_kv <= 0 || n_head <= 0 || n_kv_heads <= 0 || n_head % n_kv_heads || hb <= 0 ||
        q_rows < T || kv_rows < n_kv)
        return ROCKET_E_SHAPE;
    if (dh <= 0 || dh > 256 || dh % 8 || dv <= 0 || dv > 256 || dv % 16 || ldv % 8 || ldv < n_kv || ldo % 8)
        return ROCKET_E_UNSUPPORTED;
    const int dhp = (dh + 63) / 64;
    const int bkv = (dhp <= 2 && dv <= 128) ? 128 : 64;
    CUtensorMap tq, tk, tv;
    if (rkb::make_tmap_2d(&tq, Q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dh, static_cast<long>(n_head) * q_rows, dh, 64, BQ) ||
        rkb::make_tmap_2d(&tk, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dh, static_cast<long>(n_kv_heads) * kv_rows, dh, 64, bkv) ||
        rkb::make_tmap_2d(&tv, V, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, n_kv, static_cast<long>(n_kv_heads) * dv, ldv, 64, dv))
        return ROCKET_E_SHAPE;
    Args g;
    g.T = T; g.n_kv = n_kv; g.dv = dv; g.n_head = n_head; g.gqa = n_head / n_kv_heads;
    g.dhp = dhp; g.nkb = (n_kv + bkv - 1) / bkv;
    g.q_rows = q_rows; g.kv_rows = kv_rows; g.hb = hb; g.bstride = bstride; g.ldo = ldo;
    g.scale = scale; g.softcap = softcap;
    g.mask = static_cast<const __half *>(mask);
    g.mask_vec = mask && (n_kv % 8 == 0) && ((reinterpret_cast<uintptr_t>(mask) & 15) == 0);
    g.out = static_cast<__half *>(out);
    g.err = err;
    if (bkv == 128) launch_kind<128>(tq, tk, tv, g, stream);
    else launch_kind<64>(tq, tk, tv, g, stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "rkb flash attention launch: %s\n", cudaGetErrorString(e));
        return ROCKET_E_DEVICE;
    }
    return 0;
}

// Head-major form of the reference API: Q [n_head][T][dh], K [n_kv_heads][n_kv][dh],
// V [n_kv_heads][dv] rows of ldv elements, out [n_head][T][dv].
extern "C" int rkb_flash_attn(const void *Q, const void *K, const void *V, long ldv, const void *mask,
                              void *out, int T, int n_kv, int dh, int dv, int n_head, int n_kv_heads,
                              float scale, float softcap, int *err, cudaStream_t stream) {
    return rkb_flash_attn_ex(Q, K, V, ldv, mask, out, T, n_kv, dh, dv, n_head, n_kv_heads, scale, softcap, T,
                             n_kv, 1, static_cast<long>(T) * dv, dv, err, stream);
}
