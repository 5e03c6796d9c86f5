/*
 * rocket_matmul.h -- the matmul API of librocketnpu, B200 build.
 *
 * Every entry point below keeps the reference signature (include/rocket_matmul.h
 * of gregordinary/rocket-userspace) so ggml-rocket / tflite-rocket style callers
 * link unchanged.  Convention everywhere:
 *
 *     C[M,N] = A[M,K] * B[N,K]^T         all operands row-major
 *
 * What runs underneath is new: hand-written sm_100a kernels (tcgen05 MMA with
 * TMEM accumulators, TMA-fed multi-stage shared-memory pipelines, warp-specialised
 * producer / MMA / epilogue warps).  There is no CPU fallback: without a CUDA
 * device every compute entry returns ROCKET_E_DEVICE.
 *
 * Pointers.  A, B, C (and the scale arrays) may be host pointers (pageable or
 * pinned; the call copies in and out) or device pointers on the handle's GPU
 * (used in place, no copies).  Calls are synchronous, as in the reference.
 *
 * Shape rules are the reference's (API.md:96-104): fp16 K%32 N%16, int8 K%32
 * N%32, int4 K%32 N%64, M%4 (the one-shot entries also accept M==1).
 *
 * Numerics.
 *   int8 / int4 raw paths: exact int32 accumulation of int8 products -- bit-exact
 *     to the reference's int64 host sum whenever the result fits int32 (the
 *     reference stores (int32)sum as well, tests/matmul_int8_tiled_rocket.c:77-83).
 *   fp16: fp32 accumulation in the tensor core, one rounding to fp16 on store
 *     (tests/matmul_tiled_rocket.c:76-82 is the host definition).
 *   group-wise (int8 / int4 weights with per-(n, K-group) scales): weights are
 *     dequantised to fp16 (w * b_scale) in registers between the TMA load and the
 *     MMA and contracted with fp32 accumulation; a per-row activation scale is
 *     applied in fp32 in the epilogue.  Error against the fp64 host definition is
 *     ~1e-4 relative (two fp16 roundings), inside the 1e-2 relative-Frobenius /
 *     2e-2 max-abs bound this path is held to.
 */
#ifndef ROCKET_MATMUL_H
#define ROCKET_MATMUL_H

#include <stdint.h>
#include <stddef.h>

#ifdef ROCKET_FLOAT16_T
typedef ROCKET_FLOAT16_T _Float16;
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- tiling previews (pure, no device) ---------------------------------
 * Write the CTA tile the B200 kernel uses (Mt x Nt output tile, Kt = K-block
 * staged per pipeline step) and return the number of output tiles (> 0), or
 * ROCKET_E_SHAPE.  Reference: src/rocket_matmul.c:498-568 (fp16), :2383-2437
 * (int8), :2671-2714 (int8 group-wise), :2917 (int4). */
int rocket_matmul_plan(int M, int K, int N, int *Mt, int *Kt, int *Nt);
int rocket_matmul_plan_int8(int M, int K, int N, int *Mt, int *Kt, int *Nt);
int rocket_matmul_plan_int8_gw(int M, int K, int N, int group,
                               int *Mt, int *Kt, int *Nt);
int rocket_matmul_plan_int4(int M, int K, int N, int *Mt, int *Kt, int *Nt);

/* ---- one-shot matmuls on an open handle --------------------------------- */

/* fp16 x fp16 -> fp16, fp32 accumulate.  Replaces src/rocket_matmul.c:1945-1998. */
int rocket_matmul_fp16(int fd, int M, int K, int N,
                       const _Float16 *A, const _Float16 *B, _Float16 *C);

/* int8 x int8 -> raw int32.  Replaces src/rocket_matmul.c:2439-2627. */
int rocket_matmul_int8(int fd, int M, int K, int N,
                       const int8_t *A, const int8_t *B, int32_t *C);

/* Group-wise int8: Cf[m,n] = sum_g a_scale[m*nG+g] * b_scale[n*nG+g] * P_g[m,n],
 * P_g the exact int32 partial of K-group g, nG = K/group, group%32==0, K%group==0.
 * Replaces src/rocket_matmul.c:2716-2871. */
int rocket_matmul_int8_groupwise(int fd, int M, int K, int N,
                                 const int8_t *A, const int8_t *B,
                                 const float *a_scale, const float *b_scale,
                                 float *Cf, int group);

/* int4 values stored one per int8_t (range [-8,7]) -> raw int32.  The B200
 * kernel accumulates exactly in int32, so no int16 partial ever saturates;
 * kt_cap is accepted for ABI compatibility and does not change the result.
 * Replaces src/rocket_matmul.c:2958-3114. */
int rocket_matmul_int4(int fd, int M, int K, int N,
                       const int8_t *A, const int8_t *B, int32_t *C);
int rocket_matmul_int4_ex(int fd, int M, int K, int N,
                          const int8_t *A, const int8_t *B, int32_t *C, int kt_cap);

/* Group-wise int4 (values in [-8,7] one per int8_t), fp32 result as the int8
 * group-wise entry.  The reference's 49*group < 32767 int16 bound is kept as a
 * shape rule for compatibility.  Replaces src/rocket_matmul.c:3132-3282. */
int rocket_matmul_int4_groupwise(int fd, int M, int K, int N,
                                 const int8_t *A, const int8_t *B,
                                 const float *a_scale, const float *b_scale,
                                 float *Cf, int group);

/* fp16 x fp16 -> fp32 output (fp32 accumulate, no fp16 narrowing).
 * Replaces src/rocket_matmul.c:3620. */
int rocket_matmul_fp16_f32out(int fd, int M, int K, int N,
                              const _Float16 *A, const _Float16 *B, float *C);

/* nbatch independent same-shape fp16 matmuls C[i] = A[i] B[i]^T queued on one
 * stream with one completion wait.  Replaces src/rocket_matmul.c:2042-2330. */
int rocket_matmul_fp16_batch(int fd, int M, int K, int N, int nbatch,
                             const _Float16 *const *A, const _Float16 *const *B,
                             _Float16 *const *C);
typedef struct rocket_mm_batch rocket_mm_batch;
rocket_mm_batch *rocket_mm_batch_create(int fd);
void             rocket_mm_batch_free(rocket_mm_batch *b);
int rocket_mm_batch_run(rocket_mm_batch *b, int M, int K, int N, int nbatch,
                        const _Float16 *const *A, const _Float16 *const *B,
                        _Float16 *const *C);

/* int16 / bf16 geometry preview (K%32, N%16, M%4 or M==1). */
int rocket_matmul_plan_int16(int M, int K, int N, int *Mt, int *Kt, int *Nt);
/* Exact int16 x int16 -> int64 via four int8 GEMMs on signed hi/lo bytes;
 * inputs clamped to [-32768, 32639].  K%32, N%32.  Replaces src/rocket_matmul.c:3377. */
int rocket_matmul_int16_exact(int fd, int M, int K, int N,
                              const int16_t *A, const int16_t *B, int64_t *C);

/* bf16: fp32 A/B truncated to bf16, fp32 accumulate and output.
 * Replaces src/rocket_matmul.c:3454 and src/rocket_bf16_stream.c. */
int rocket_matmul_plan_bf16(int M, int K, int N, int *Mt, int *Kt, int *Nt);
int rocket_matmul_bf16(int fd, int M, int K, int N, const float *A, const float *B, float *C);
int rocket_matmul_bf16_mt(int M, int K, int N, const float *A, const float *B, float *C, int nthreads);
typedef struct rocket_bf16_stream rocket_bf16_stream;
rocket_bf16_stream *rocket_bf16_stream_create(int nthreads);
void                rocket_bf16_stream_free(rocket_bf16_stream *s);
int rocket_matmul_bf16_stream(rocket_bf16_stream *s, int M, int K, int N,
                              const float *A, const float *B, float *C);

/* tf32: fp32 A/B fed to the tf32 tensor-core path, fp32 accumulate and output.
 * K%16, N%16.  Replaces src/rocket_matmul.c:3840. */
int rocket_matmul_plan_tf32(int M, int K, int N, int *Mt, int *Kt, int *Nt);
int rocket_matmul_tf32(int fd, int M, int K, int N, const float *A, const float *B, float *C);

/* ---- multi-GPU fan-out ---------------------------------------------------
 * Split N across `nthreads` GPUs (clamped to [1, 8] and to the visible device
 * count; nthreads > devices wraps round-robin), one host worker thread per
 * slice, each slice C[:, n0:n1] computed on its own device and copied into C.
 * Slices are multiples of 16 columns.  Replaces src/rocket_matmul_mt.c:58-99. */
int rocket_matmul_fp16_mt(int M, int K, int N,
                          const _Float16 *A, const _Float16 *B, _Float16 *C,
                          int nthreads);

/* ---- resident fp16 weights ------------------------------------------------
 * A ctx owns one worker per GPU slice; rocket_weights_pack uploads each
 * worker's N-slice of B once; each prepacked call then moves only A and C.
 * The resident layout is M-independent, so one pack serves every M.  K and N
 * must match the pack (else ROCKET_E_SHAPE).  Free weights before the ctx.  Not
 * thread-safe per ctx.  Replaces src/rocket_prepacked.c:106-447. */
typedef struct rocket_ctx     rocket_ctx;
typedef struct rocket_weights rocket_weights;

rocket_ctx     *rocket_ctx_create(int nthreads);
void            rocket_ctx_free(rocket_ctx *ctx);
rocket_weights *rocket_weights_pack(rocket_ctx *ctx, int M, int K, int N, const _Float16 *B);
void            rocket_weights_free(rocket_ctx *ctx, rocket_weights *w);
int rocket_matmul_fp16_prepacked(rocket_ctx *ctx, int M, int K, int N,
                                 const _Float16 *A, _Float16 *C, rocket_weights *w);

/* ---- streaming fp16: weights re-uploaded every call ------------------------
 * A stream keeps its workers (GPUs) and weight buffers across calls; each call
 * uploads this call's B (or, fused, the N-concatenation of nseg weights that
 * share A -- QKV, gate+up) and runs the N-split matmul.  C of the fused form is
 * [M, sum Ns].  Not thread-safe per stream.  Replaces src/rocket_prepacked.c:459-505. */
#define ROCKET_MAX_FUSE 8
typedef struct rocket_stream rocket_stream;
rocket_stream *rocket_stream_create(int nthreads);
void           rocket_stream_free(rocket_stream *s);
int rocket_matmul_fp16_stream(rocket_stream *s, int M, int K, int N,
                              const _Float16 *A, const _Float16 *B, _Float16 *C);
int rocket_matmul_fp16_stream_fused(rocket_stream *s, int M, int K,
                                    const _Float16 *const *Bs, const int *Ns, int nseg,
                                    const _Float16 *A, _Float16 *C);

/* ---- resident int8 (W8A8) --------------------------------------------------
 * Per-channel form returns raw int32, group-wise form the fp32 scaled sum.
 * N-slices are multiples of 32 columns.  Replaces src/rocket_prepacked_int8.c
 * :167-767. */
typedef struct rocket_i8_ctx     rocket_i8_ctx;
typedef struct rocket_i8_weights rocket_i8_weights;

rocket_i8_ctx     *rocket_i8_ctx_create(int nthreads);
void               rocket_i8_ctx_free(rocket_i8_ctx *ctx);
rocket_i8_weights *rocket_i8_weights_pack(rocket_i8_ctx *ctx, int M, int K, int N,
                                          const int8_t *B);
rocket_i8_weights *rocket_i8_weights_pack_gw(rocket_i8_ctx *ctx, int M, int K, int N,
                                             const int8_t *B, int group);
void               rocket_i8_weights_free(rocket_i8_ctx *ctx, rocket_i8_weights *w);
/* Device bytes held by the packed weight (all slices). */
size_t             rocket_i8_weights_bytes(const rocket_i8_weights *w);
int rocket_matmul_int8_prepacked(rocket_i8_ctx *ctx, int M, int K, int N,
                                 const int8_t *A, int32_t *C, rocket_i8_weights *w);
int rocket_matmul_int8_prepacked_gw(rocket_i8_ctx *ctx, int M, int K, int N,
                                    const int8_t *A, const float *a_scale,
                                    const float *b_scale, float *Cf, rocket_i8_weights *w);

/* ---- resident int4 ----------------------------------------------------------
 * Weights are held nibble-packed on the device (two int4 per byte, half the
 * int8 footprint) in 256-row x K-block tiles; kernels unpack them in registers.
 * N-slices are multiples of 64 columns.  A may use the full int8 range, so the
 * group-wise form also serves W4A8.  Replaces src/rocket_prepacked_int4.c
 * :122-686. */
typedef struct rocket_i4_ctx     rocket_i4_ctx;
typedef struct rocket_i4_weights rocket_i4_weights;

rocket_i4_ctx     *rocket_i4_ctx_create(int nthreads);
void               rocket_i4_ctx_free(rocket_i4_ctx *ctx);
rocket_i4_weights *rocket_i4_weights_pack(rocket_i4_ctx *ctx, int M, int K, int N,
                                          const int8_t *B);
rocket_i4_weights *rocket_i4_weights_pack_gw(rocket_i4_ctx *ctx, int M, int K, int N,
                                             const int8_t *B, int group);
void               rocket_i4_weights_free(rocket_i4_ctx *ctx, rocket_i4_weights *w);
size_t             rocket_i4_weights_bytes(const rocket_i4_weights *w);
int rocket_matmul_int4_prepacked(rocket_i4_ctx *ctx, int M, int K, int N,
                                 const int8_t *A, int32_t *C, rocket_i4_weights *w);
int rocket_matmul_int4_prepacked_gw(rocket_i4_ctx *ctx, int M, int K, int N,
                                    const int8_t *A, const float *a_scale,
                                    const float *b_scale, float *Cf, rocket_i4_weights *w);

#ifdef __cplusplus
}
#endif
#endif /* ROCKET_MATMUL_H */
