// rowops.cu -- the HBM-bound encoder ops: LayerNorm / RMSNorm, softmax /
// log-softmax, the activation zoo, element-wise add / mul / sub, the gated
// product act(gate) * up, and the head split that feeds the attention kernel.
//
// Replaces the reference's composed NPU programs (src/rocket_norm.c:152-227,
// src/rocket_softmax.c:38-78, src/rocket_activation.c, src/rocket_ffn.c:23-50),
// which build each of these from LUT passes, element-wise passes and
// ones-matmul reductions with host tails.  Here each op is one pass over HBM:
// a warp owns a row (norms, softmax) and reduces with shuffles; element-wise
// ops move 16 bytes per thread per step.  All arithmetic is fp32 on fp16
// storage; reductions are exact-order independent to within fp32 rounding.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <type_traits>
#include <stdint.h>
#include "../src/rkb_kernels.h"
#include "../../include/rocket_npu.h"

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Row loads as 8-half vectors when the row is 16-byte aligned, else scalar.
struct RowView {
    const __half *p;
    int n;
    bool vec;
};

template <class F>
__device__ __forceinline__ void row_for_each(const RowView &r, int lane, F f) {
    if (r.vec) {
        const int nv = r.n >> 3;
        for (int i = lane; i < nv; i += 32) {
            uint4 u = reinterpret_cast<const uint4 *>(r.p)[i];
            const __half *h = reinterpret_cast<const __half *>(&u);
#pragma unroll
            for (int j = 0; j < 8; ++j) f(i * 8 + j, __half2float(h[j]));
        }
    } else {
        for (int i = lane; i < r.n; i += 32) f(i, __half2float(r.p[i]));
    }
}

// Rows of up to 32 * 8 * NVR halves (16-byte aligned, H % 8 == 0): one read
// into registers, the same two-pass statistics as norm_rows (same summation
// order, so the same results), one write.  NVR is sized to H so the register
// footprint -- and the occupancy an HBM-bound kernel needs -- follows the row.
template <int NVR>
__global__ void norm_rows_reg(const __half *__restrict__ x, const __half *__restrict__ gamma,
                              const __half *__restrict__ beta, int M, int H, float eps, int mode,
                              __half *__restrict__ out) {
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nv = H >> 3;
    for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(row) * H);
        uint4 u[NVR];
#pragma unroll
        for (int k = 0; k < NVR; ++k)
            if (lane + 32 * k < nv) u[k] = src[lane + 32 * k];
        float mean = 0.f;
        if (mode == 0) {
            float sm = 0.f;
#pragma unroll
            for (int k = 0; k < NVR; ++k)
                if (lane + 32 * k < nv) {
                    const __half *h = reinterpret_cast<const __half *>(&u[k]);
#pragma unroll
                    for (int j = 0; j < 8; ++j) sm += __half2float(h[j]);
                }
            mean = warp_sum(sm) / H;
        }
        float qs = 0.f;
#pragma unroll
        for (int k = 0; k < NVR; ++k)
            if (lane + 32 * k < nv) {
                const __half *h = reinterpret_cast<const __half *>(&u[k]);
#pragma unroll
                for (int j = 0; j < 8; ++j) { const float dd = __half2float(h[j]) - mean; qs += dd * dd; }
            }
        const float rstd = rsqrtf(warp_sum(qs) / H + eps);
        uint4 *dst = reinterpret_cast<uint4 *>(out + static_cast<size_t>(row) * H);
#pragma unroll
        for (int k = 0; k < NVR; ++k) {
            const int i = lane + 32 * k;
            if (i >= nv) continue;
            const uint4 g = reinterpret_cast<const uint4 *>(gamma)[i];
            const uint4 b = beta ? reinterpret_cast<const uint4 *>(beta)[i] : make_uint4(0, 0, 0, 0);
            const __half *h = reinterpret_cast<const __half *>(&u[k]);
            const __half *gh = reinterpret_cast<const __half *>(&g);
            const __half *bh = reinterpret_cast<const __half *>(&b);
            uint4 w;
            __half *wh = reinterpret_cast<__half *>(&w);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                wh[j] = __float2half_rn((__half2float(h[j]) - mean) * rstd * __half2float(gh[j]) +
                                        __half2float(bh[j]));
            dst[i] = w;
        }
    }
}

// mode 0: LayerNorm (gamma, optional beta), mode 1: RMSNorm (weight = gamma)
__global__ void norm_rows(const __half *__restrict__ x, const __half *__restrict__ gamma,
                          const __half *__restrict__ beta, int M, int H, float eps, int mode,
                          __half *__restrict__ out) {
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    const bool vec = (H % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
    for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
        RowView r{x + static_cast<size_t>(row) * H, H, vec};
        float mean = 0.f;
        if (mode == 0) {
            float s = 0.f;
            row_for_each(r, lane, [&](int, float v) { s += v; });
            mean = warp_sum(s) / H;
        }
        float q = 0.f;
        row_for_each(r, lane, [&](int, float v) { const float d = v - mean; q += d * d; });
        const float rstd = rsqrtf(warp_sum(q) / H + eps);
        __half *o = out + static_cast<size_t>(row) * H;
        if (vec) {
            const int nv = H >> 3;
            for (int i = lane; i < nv; i += 32) {
                uint4 u = reinterpret_cast<const uint4 *>(r.p)[i];
                uint4 g = reinterpret_cast<const uint4 *>(gamma)[i];
                uint4 b = beta ? reinterpret_cast<const uint4 *>(beta)[i] : make_uint4(0, 0, 0, 0);
                const __half *h = reinterpret_cast<const __half *>(&u);
                const __half *gh = reinterpret_cast<const __half *>(&g);
                const __half *bh = reinterpret_cast<const __half *>(&b);
                uint4 w;
                __half *wh = reinterpret_cast<__half *>(&w);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    wh[j] = __float2half_rn((__half2float(h[j]) - mean) * rstd * __half2float(gh[j]) +
                                            __half2float(bh[j]));
                reinterpret_cast<uint4 *>(o)[i] = w;
            }
        } else {
            for (int i = lane; i < H; i += 32) {
                const float b = beta ? __half2float(beta[i]) : 0.f;
                o[i] = __float2half_rn((__half2float(r.p[i]) - mean) * rstd * __half2float(gamma[i]) + b);
            }
        }
    }
}

// mode 0: softmax, mode 1: log-softmax
__global__ void softmax_rows(const __half *__restrict__ x, int M, int N, int mode,
                             __half *__restrict__ out) {
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    const bool vec = (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
    for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
        RowView r{x + static_cast<size_t>(row) * N, N, vec};
        float mx = -INFINITY;
        row_for_each(r, lane, [&](int, float v) { mx = fmaxf(mx, v); });
        mx = warp_max(mx);
        float s = 0.f;
        row_for_each(r, lane, [&](int, float v) { s += expf(v - mx); });
        s = warp_sum(s);
        const float inv = 1.f / s, lse = mx + logf(s);
        __half *o = out + static_cast<size_t>(row) * N;
        if (vec) {
            const int nv = N >> 3;
            for (int i = lane; i < nv; i += 32) {
                uint4 u = reinterpret_cast<const uint4 *>(r.p)[i];
                const __half *h = reinterpret_cast<const __half *>(&u);
                uint4 w;
                __half *wh = reinterpret_cast<__half *>(&w);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float v = __half2float(h[j]);
                    wh[j] = __float2half_rn(mode ? v - lse : expf(v - mx) * inv);
                }
                reinterpret_cast<uint4 *>(o)[i] = w;
            }
        } else {
            for (int i = lane; i < N; i += 32) {
                const float v = __half2float(r.p[i]);
                o[i] = __float2half_rn(mode ? v - lse : expf(v - mx) * inv);
            }
        }
    }
}

// Softmax / log-softmax with the row held in registers: one HBM read and one
// write per element, one exponential per element (rows of up to 32 * MAXE
// halves).  V halves per load (16 / 8 / 4 / 2 bytes), chosen by the caller
// from N and the pointers' alignment, so odd-sized rows (1500 in the config-4
// attention) still load whole vectors.  Element e of chunk c of a lane is row
// index (c * 32 + lane) * V + e; indices past N hold -inf (weight 0).
template <int V, int MAXE>
__global__ void __launch_bounds__(128, 4) softmax_rows_reg(const __half *__restrict__ x, int M, int N, int mode,
                                 __half *__restrict__ out) {
    constexpr int MAXC = MAXE / V;
    using Vec = typename std::conditional<V == 8, uint4, typename std::conditional<V == 4, uint2,
                typename std::conditional<V == 2, uint32_t, uint16_t>::type>::type>::type;
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nch = (N + 32 * V - 1) / (32 * V);
    for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
        const Vec *src = reinterpret_cast<const Vec *>(x + static_cast<size_t>(row) * N);
        // all of the row's loads are issued before any is used
        Vec raw[MAXC];
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
            const int i = c * 32 + lane;
            if (c < nch && i * V < N) raw[c] = __ldcs(src + i);
        }
        // the row stays as fp16 in registers; the exponential is evaluated
        // again for the output instead of keeping fp32 copies (half the
        // registers, so twice the rows in flight per SM)
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
            const bool in = c < nch && (c * 32 + lane) * V < N;
            const __half *h = reinterpret_cast<const __half *>(&raw[c]);
#pragma unroll
            for (int e = 0; e < V; ++e)
                if (in) mx = fmaxf(mx, __half2float(h[e]));
        }
        mx = warp_max(mx);
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
            const bool in = c < nch && (c * 32 + lane) * V < N;
            const __half *h = reinterpret_cast<const __half *>(&raw[c]);
#pragma unroll
            for (int e = 0; e < V; ++e)
                if (in) sum += __expf(__half2float(h[e]) - mx);
        }
        sum = warp_sum(sum);
        const float inv = 1.f / sum, lse = mx + __logf(sum);
        Vec *dst = reinterpret_cast<Vec *>(out + static_cast<size_t>(row) * N);
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
            const int i = c * 32 + lane;
            if (c < nch && i * V < N) {
                const __half *h = reinterpret_cast<const __half *>(&raw[c]);
                Vec w;
                __half *wh = reinterpret_cast<__half *>(&w);
#pragma unroll
                for (int e = 0; e < V; ++e) {
                    const float xv = __half2float(h[e]);
                    wh[e] = __float2half_rn(mode ? xv - lse : __expf(xv - mx) * inv);
                }
                __stcs(dst + i, w);
            }
        }
    }
}

// Activation kinds follow the reference enum (include/rocket_activation.h:48-135);
// definitions follow its exact host evaluation (src/rocket_activation.c:48-77).
__device__ __forceinline__ float act_eval(int kind, float x) {
    switch (kind) {
    case 0: return 1.f / (1.f + expf(-x));                                   // sigmoid
    case 1: return fminf(fmaxf(x / 6.f + 0.5f, 0.f), 1.f);                   // hardsigmoid
    case 2: return x * fminf(fmaxf(x / 6.f + 0.5f, 0.f), 1.f);               // hardswish
    case 3: return x / (1.f + expf(-x));                                     // silu
    case 4: return tanhf(x);
    case 5: return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));        // gelu (erf)
    case 7: return x > 0.f ? sqrtf(x) : 0.f;
    case 8: return x > 0.f ? rsqrtf(x) : 0.f;
    case 9: return x != 0.f ? 1.f / x : 0.f;
    case 10: return expf(x);
    case 11: return 0.5f * (1.f + erff(x * 0.70710678118654752f));           // gelu gate (Phi)
    case 12: return x > 0.f ? x + log1pf(expf(-x)) : log1pf(expf(x));        // softplus
    case 13: return tanhf(x > 0.f ? x + log1pf(expf(-x)) : log1pf(expf(x))); // mish gate
    case 14: return x * tanhf(x > 0.f ? x + log1pf(expf(-x)) : log1pf(expf(x)));
    case 15: return fabsf(x);
    case 18: return x > 0.f ? logf(x) : 0.f;
    default: return 0.f;
    }
}

// op: 0 act(a), 1 a+b, 2 a*b, 3 a-b, 4 act(a)*b, 5 max(a,b), 6 min(a,b),
// 7 clip(a, lo, hi).  The op is a template parameter so each kernel's inner
// loop is branch-free; 16-byte loads and stores (8 halves) per thread.
template <int OP>
__device__ __forceinline__ float ew_eval(int kind, float x, float y, float lo, float hi) {
    if (OP == 0) return act_eval(kind, x);
    if (OP == 1) return x + y;
    if (OP == 2) return x * y;
    if (OP == 3) return x - y;
    if (OP == 4) return act_eval(kind, x) * y;
    if (OP == 5) return fmaxf(x, y);
    if (OP == 6) return fminf(x, y);
    return fminf(fmaxf(x, lo), hi);
}

template <int OP>
__global__ void elementwise(const __half *__restrict__ a, const __half *__restrict__ b, int kind,
                            float lo, float hi, size_t n, __half *__restrict__ out) {
    constexpr bool TWO = OP >= 1 && OP <= 6;
    const size_t nv = n / 8;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nv; i += stride) {
        uint4 ua = reinterpret_cast<const uint4 *>(a)[i];
        uint4 ub = TWO ? reinterpret_cast<const uint4 *>(b)[i] : make_uint4(0, 0, 0, 0);
        const __half *ha = reinterpret_cast<const __half *>(&ua);
        const __half *hb = reinterpret_cast<const __half *>(&ub);
        uint4 w;
        __half *wh = reinterpret_cast<__half *>(&w);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            wh[j] = __float2half_rn(ew_eval<OP>(kind, __half2float(ha[j]), __half2float(hb[j]), lo, hi));
        reinterpret_cast<uint4 *>(out)[i] = w;
    }
    for (size_t i = nv * 8 + blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
        const float x = __half2float(a[i]), y = TWO ? __half2float(b[i]) : 0.f;
        out[i] = __float2half_rn(ew_eval<OP>(kind, x, y, lo, hi));
    }
}

// qkv [B*T, 3d] (q | k | v column blocks) -> per head, zero-padded to Tp rows:
//   Q [B*H, Tp, dh], K [B*H, Tp, dh], Vt [B*H, dh, Tp]
__global__ void split_heads(const __half *__restrict__ qkv, long ld, int B, int T, int Tp, int H,
                            int dh, __half *__restrict__ Q, __half *__restrict__ K,
                            __half *__restrict__ Vt) {
    // one thread per (b, h, t, 8-wide chunk of dh)
    const int cpr = dh / 8;
    const size_t total = static_cast<size_t>(B) * H * Tp * cpr;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % cpr);
        const int t = static_cast<int>((i / cpr) % Tp);
        const int bh = static_cast<int>(i / (static_cast<size_t>(cpr) * Tp));
        const int b = bh / H, h = bh % H;
        uint4 q = make_uint4(0, 0, 0, 0), k = q, v = q;
        if (t < T) {
            const __half *row = qkv + static_cast<size_t>(b * T + t) * ld + h * dh + c * 8;
            const int d = H * dh;
            q = *reinterpret_cast<const uint4 *>(row);
            k = *reinterpret_cast<const uint4 *>(row + d);
            v = *reinterpret_cast<const uint4 *>(row + 2 * d);
        }
        const size_t qo = (static_cast<size_t>(bh) * Tp + t) * dh + c * 8;
        *reinterpret_cast<uint4 *>(Q + qo) = q;
        *reinterpret_cast<uint4 *>(K + qo) = k;
        const __half *vh = reinterpret_cast<const __half *>(&v);
        __half *vt = Vt + static_cast<size_t>(bh) * dh * Tp;
#pragma unroll
        for (int j = 0; j < 8; ++j) vt[static_cast<size_t>(c * 8 + j) * Tp + t] = vh[j];
    }
}

// The same split, one CTA per (64-token tile, batch x head): Q and K rows are
// copied with 16-byte loads and stores, and V goes through shared memory so
// that every V^T row segment (64 tokens = 128 bytes) is written with 16-byte
// stores instead of scattered 2-byte ones.  Tp % 64 == 0, dh % 8 == 0, dh <= 256.
__global__ void __launch_bounds__(256) split_heads_tiled(const __half *__restrict__ qkv, long ld, int T,
                                                         int Tp, int H, int dh, __half *__restrict__ Q,
                                                         __half *__restrict__ K, __half *__restrict__ Vt) {
    extern __shared__ __align__(16) __half sv[];           // [64 tokens][dh + 8]
    const int pitch = dh + 8;                                // 16-byte shift per row: fewer bank conflicts
    const int t0 = blockIdx.x * 64, bh = blockIdx.y;
    const int b = bh / H, h = bh % H;
    const int cpr = dh / 8, d = H * dh;
    for (int i = threadIdx.x; i < 64 * cpr; i += blockDim.x) {
        const int tl = i / cpr, c = i % cpr, t = t0 + tl;
        uint4 q = make_uint4(0, 0, 0, 0), k = q, v = q;
        if (t < T) {
            const __half *row = qkv + static_cast<size_t>(b * T + t) * ld + h * dh + c * 8;
            q = *reinterpret_cast<const uint4 *>(row);
            k = *reinterpret_cast<const uint4 *>(row + d);
            v = *reinterpret_cast<const uint4 *>(row + 2 * d);
        }
        const size_t qo = (static_cast<size_t>(bh) * Tp + t) * dh + c * 8;
        *reinterpret_cast<uint4 *>(Q + qo) = q;
        *reinterpret_cast<uint4 *>(K + qo) = k;
        *reinterpret_cast<uint4 *>(sv + tl * pitch + c * 8) = v;
    }
    __syncthreads();
    __half *vt = Vt + static_cast<size_t>(bh) * dh * Tp + t0;
    for (int i = threadIdx.x; i < dh * 8; i += blockDim.x) {
        const int dd = i / 8, tc = i % 8;                    // feature row, 8-token chunk
        uint4 w;
        __half *wh = reinterpret_cast<__half *>(&w);
#pragma unroll
        for (int j = 0; j < 8; ++j) wh[j] = sv[(tc * 8 + j) * pitch + dd];
        *reinterpret_cast<uint4 *>(vt + static_cast<size_t>(dd) * Tp + tc * 8) = w;
    }
}

// out[m] = sum (or mean) of row m, fp32 (src/rocket_reduce.c:380-390 definition)
__global__ void reduce_rows(const __half *__restrict__ x, int M, int H, int mean, float *__restrict__ out) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (H % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
        RowView r{x + static_cast<size_t>(row) * H, H, vec};
        float s = 0.f;
        row_for_each(r, lane, [&](int, float v) { s += v; });
        s = warp_sum(s);
        if (lane == 0) out[row] = mean ? s / H : s;
    }
}

// Inclusive / exclusive, forward / reverse prefix sums per row (fp32 running
// sum, fp16 store): one warp per row, 32-element chunks, shuffle scan + carry
// (src/rocket_reduce.c:445-464 definition).
__global__ void cumsum_rows(const __half *__restrict__ x, int M, int N, int exclusive, int reverse,
                            __half *__restrict__ out) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
        const __half *xr = x + static_cast<size_t>(row) * N;
        __half *orow = out + static_cast<size_t>(row) * N;
        float carry = 0.f;
        for (int base = 0; base < N; base += 32) {
            const int j = base + lane;
            const int idx = reverse ? N - 1 - j : j;
            const float v = (j < N) ? __half2float(xr[idx]) : 0.f;
            float incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            if (j < N) orow[idx] = __float2half_rn(carry + (exclusive ? incl - v : incl));
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
}

// out[m, n] = in[m, n] * r[m] (src/rocket_norm.c:21-30 definition)
__global__ void scale_rows(const __half *__restrict__ x, const float *__restrict__ r, int M, int N,
                           __half *__restrict__ out) {
    const size_t total = static_cast<size_t>(M) * N;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = __float2half_rn(__half2float(x[i]) * r[i / N]);
}

// loss[m] = logsumexp(row m) - row[m][target[m]] (src/rocket_softmax.c:141-155 definition)
__global__ void cross_entropy_rows(const __half *__restrict__ x, const int *__restrict__ target, int M,
                                   int N, float *__restrict__ loss) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
        RowView r{x + static_cast<size_t>(row) * N, N, vec};
        float mx = -INFINITY;
        row_for_each(r, lane, [&](int, float v) { mx = fmaxf(mx, v); });
        mx = warp_max(mx);
        float s = 0.f;
        row_for_each(r, lane, [&](int, float v) { s += expf(v - mx); });
        s = warp_sum(s);
        if (lane == 0) {
            const int t = target[row];
            const float g = (t >= 0 && t < N) ? __half2float(r.p[t]) : 0.f;
            loss[row] = mx + logf(s) - g;
        }
    }
}

int grid_for(size_t work, int threads) {
    size_t b = (work + threads - 1) / threads;
    if (b > 148 * 32) b = 148 * 32;
    return b < 1 ? 1 : static_cast<int>(b);
}
int status() { return cudaGetLastError() == cudaSuccess ? 0 : ROCKET_E_DEVICE; }

}  // namespace

extern "C" {

int rkb_norm_rows(const void *x, const void *gamma, const void *beta, int M, int H, float eps,
                  int rms, void *out, cudaStream_t s) {
    if (M <= 0 || H <= 0 || !gamma) return ROCKET_E_SHAPE;
    const int warps = 8;
    int grid = (M + warps - 1) / warps;
    if (grid > 148 * 16) grid = 148 * 16;
    const bool vec = H % 8 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                                     reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0;
    const __half *xh = static_cast<const __half *>(x), *gh = static_cast<const __half *>(gamma),
                 *bh = static_cast<const __half *>(beta);
    __half *oh = static_cast<__half *>(out);
    const int mode = rms ? 1 : 0;
    if (vec && H <= 512)
        norm_rows_reg<2><<<grid, warps * 32, 0, s>>>(xh, gh, bh, M, H, eps, mode, oh);
    else if (vec && H <= 1024)
        norm_rows_reg<4><<<grid, warps * 32, 0, s>>>(xh, gh, bh, M, H, eps, mode, oh);
    else if (vec && H <= 2048)
        norm_rows_reg<8><<<grid, warps * 32, 0, s>>>(xh, gh, bh, M, H, eps, mode, oh);
    else
        norm_rows<<<grid, warps * 32, 0, s>>>(xh, gh, bh, M, H, eps, mode, oh);
    return status();
}

int rkb_softmax_rows(const void *x, int M, int N, int log_mode, void *out, cudaStream_t s) {
    if (M <= 0 || N <= 0) return ROCKET_E_SHAPE;
    const int warps = 8;
    int grid = (M + warps - 1) / warps;
    if (grid > 148 * 16) grid = 148 * 16;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out);
    const __half *hx = static_cast<const __half *>(x);
    __half *ho = static_cast<__half *>(out);
    const int m = log_mode ? 1 : 0;
    if (N <= 32 * 64) {
        const int v = (N % 8 == 0 && (al & 15) == 0) ? 8 : (N % 4 == 0 && (al & 7) == 0) ? 4
                    : (N % 2 == 0 && (al & 3) == 0) ? 2 : 1;
        // per-lane row share, rounded to the next instantiated size (whole V-vectors)
        const int need = ((N + 32 * v - 1) / (32 * v)) * v;
        const int e = need <= 8 ? 8 : need <= 16 ? 16 : need <= 32 ? 32 : need <= 48 ? 48 : 64;
        // 4-warp blocks: finer occupancy steps for these register-heavy rows
        int grid4 = (M + 3) / 4;
        if (grid4 > 148 * 32) grid4 = 148 * 32;
        const dim3 gr(grid4), bl(128);
#define RKB_SMX(V, E) softmax_rows_reg<V, E><<<gr, bl, 0, s>>>(hx, M, N, m, ho)
#define RKB_SMX_E(V) do { if (e == 8) RKB_SMX(V, 8); else if (e == 16) RKB_SMX(V, 16); \
                          else if (e == 32) RKB_SMX(V, 32); else if (e == 48) RKB_SMX(V, 48); \
                          else RKB_SMX(V, 64); } while (0)
        if (v == 8) RKB_SMX_E(8);
        else if (v == 4) RKB_SMX_E(4);
        else if (v == 2) RKB_SMX_E(2);
        else RKB_SMX_E(1);
#undef RKB_SMX_E
#undef RKB_SMX
        return status();
    }
    softmax_rows<<<grid, warps * 32, 0, s>>>(static_cast<const __half *>(x), M, N, log_mode ? 1 : 0,
                                             static_cast<__half *>(out));
    return status();
}

int rkb_elementwise(const void *a, const void *b, int op, int kind, size_t n, void *out,
                    cudaStream_t s) {
    return rkb_elementwise_ex(a, b, op, kind, 0.f, 0.f, n, out, s);
}

int rkb_elementwise_ex(const void *a, const void *b, int op, int kind, float lo, float hi, size_t n,
                       void *out, cudaStream_t s) {
    if (n == 0 || op < 0 || op > 7) return ROCKET_E_SHAPE;
    if ((op >= 1 && op <= 6) && !b) return ROCKET_E_SHAPE;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
         reinterpret_cast<uintptr_t>(out)) & 15)
        return ROCKET_E_SHAPE;
    const __half *ha = static_cast<const __half *>(a), *hb = static_cast<const __half *>(b);
    __half *ho = static_cast<__half *>(out);
    const int grid = grid_for(n / 8 + 1, 256);
    switch (op) {
    case 0: elementwise<0><<<grid, 256, 0, s>>>(ha, hb, kind, lo, hi, n, ho); break;
    case 1: elementwise<1><<<grid, 256, 0, s>>>(ha, hb, kind, lo, hi, n, ho); break;
    case 2: elementwise<2><<<grid, 256, 0, s>>>(ha, hb, kind, lo, hi, n, ho); break;
    case 3: elementwise<3><<<grid, 256, 0, s>>>(ha, hb, kind, lo, hi, n, ho); break;
    case 4: elementwise<4><<<grid, 256, 0, s>>>(ha, hb, kind, lo, hi, n, ho); break;
    case 5: elementwise<5><<<grid, 256, 0, s>>>(ha, hb, kind, lo, hi, n, ho); break;
    case 6: elementwise<6><<<grid, 256, 0, s>>>(ha, hb, kind, lo, hi, n, ho); break;
    default: elementwise<7><<<grid, 256, 0, s>>>(ha, hb, kind, lo, hi, n, ho); break;
    }
    return status();
}

int rkb_reduce_rows(const void *x, int M, int H, int mean, float *out, cudaStream_t s) {
    if (M <= 0 || H <= 0) return ROCKET_E_SHAPE;
    int grid = (M + 7) / 8;
    if (grid > 148 * 16) grid = 148 * 16;
    reduce_rows<<<grid, 256, 0, s>>>(static_cast<const __half *>(x), M, H, mean, out);
    return status();
}

int rkb_cumsum_rows(const void *x, int M, int N, int exclusive, int reverse, void *out, cudaStream_t s) {
    if (M <= 0 || N <= 0) return ROCKET_E_SHAPE;
    int grid = (M + 7) / 8;
    if (grid > 148 * 16) grid = 148 * 16;
    cumsum_rows<<<grid, 256, 0, s>>>(static_cast<const __half *>(x), M, N, exclusive, reverse,
                                     static_cast<__half *>(out));
    return status();
}

int rkb_scale_rows(const void *x, const float *r, int M, int N, void *out, cudaStream_t s) {
    if (M <= 0 || N <= 0) return ROCKET_E_SHAPE;
    scale_rows<<<grid_for(static_cast<size_t>(M) * N, 256), 256, 0, s>>>(static_cast<const __half *>(x), r, M, N,
                                                                          static_cast<__half *>(out));
    return status();
}

int rkb_cross_entropy_rows(const void *x, const int *target, int M, int N, float *loss, cudaStream_t s) {
    if (M <= 0 || N <= 0) return ROCKET_E_SHAPE;
    int grid = (M + 7) / 8;
    if (grid > 148 * 16) grid = 148 * 16;
    cross_entropy_rows<<<grid, 256, 0, s>>>(static_cast<const __half *>(x), target, M, N, loss);
    return status();
}

int rkb_split_heads(const void *qkv, long ld, int B, int T, int Tp, int H, int dh, void *Q, void *K,
                    void *Vt, cudaStream_t s) {
    if (dh % 8 || (ld % 8)) return ROCKET_E_SHAPE;
    if (Tp % 64 == 0 && dh <= 256 && (reinterpret_cast<uintptr_t>(qkv) & 15) == 0 &&
        static_cast<long>(B) * H <= 65535) {
        const size_t smem = 64 * static_cast<size_t>(dh + 8) * 2;
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(split_heads_tiled, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        split_heads_tiled<<<dim3(Tp / 64, B * H), 256, smem, s>>>(
            static_cast<const __half *>(qkv), ld, T, Tp, H, dh, static_cast<__half *>(Q),
            static_cast<__half *>(K), static_cast<__half *>(Vt));
        return status();
    }
    const size_t total = static_cast<size_t>(B) * H * Tp * (dh / 8);
    split_heads<<<grid_for(total, 256), 256, 0, s>>>(static_cast<const __half *>(qkv), ld, B, T, Tp, H, dh,
                                                     static_cast<__half *>(Q), static_cast<__half *>(K),
                                                     static_cast<__half *>(Vt));
    return status();
}

}  // extern "C"
