/*
 * rocket_b200.h -- B200-only extensions of librocketnpu.  None of these has a
 * counterpart in the reference API; a caller that only uses rocket_npu.h and
 * rocket_matmul.h never needs them.  They expose what a GPU caller wants on
 * top of the synchronous reference API: the CUDA stream a handle runs on (to
 * order its own work or record events), and per-kernel device timing.
 */
#ifndef ROCKET_B200_H
#define ROCKET_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The cudaStream_t (as void*) of an open handle, NULL if fd is not open. */
void *rocket_b200_stream(int fd);
/* The CUDA device ordinal of an open handle, or ROCKET_E_DEVICE. */
int   rocket_b200_device(int fd);
/* The handle of worker `worker` of a rocket_ctx / rocket_i8_ctx / rocket_i4_ctx
 * (all three share one layout), or ROCKET_E_SHAPE when out of range. */
int   rocket_b200_ctx_fd(const void *ctx, int worker);

/* Deferred completion for this host thread.  The reference API is synchronous
 * and stays so by default.  With rocket_b200_set_async(1), a dense or
 * per-channel resident matmul whose operands are ALL device memory on the
 * worker GPUs (nothing to copy to or from the host) returns right after its
 * kernels are enqueued on the handle's stream; its status -- including a
 * bounded-wait expiry inside a kernel -- is returned by the next
 * rocket_b200_sync(fd) / rocket_b200_ctx_sync(ctx).  Calls that stage host
 * memory, and the group-wise entries, still wait before returning.  Work on
 * one handle runs in call order, so back-to-back calls queue without gaps. */
void  rocket_b200_set_async(int on);
int   rocket_b200_sync(int fd);
int   rocket_b200_ctx_sync(const void *ctx);

/* Kernel profiling (the device-side analogue of the reference's
 * ROCKET_MM_PROFILE, src/rocket_matmul.c:74-125).  While enabled (also by the
 * environment variable ROCKET_MM_PROFILE=1), every kernel the library launches
 * is bracketed by CUDA events on its own stream; the elapsed times are
 * accumulated per kernel family when the call completes.  Families are
 * indexed 0..n-1; get returns 0, or ROCKET_E_SHAPE past the last one. */
void  rocket_b200_profile_enable(int on);
void  rocket_b200_profile_reset(void);
int   rocket_b200_profile_get(int idx, const char **name, uint64_t *launches, double *total_ms);

/* Group-wise int4 matmul that allocates nothing.  No counterpart in the
 * reference.  For callers that may not call cudaMalloc (a runtime that owns all
 * device memory through its own arena, a fixed memory budget, or a loop that
 * must not allocate while it runs): rocket_matmul_int4_groupwise's inputs and
 * output, computed in the fast group-wise form (as rocket_b200_gw_mode(1):
 * w * b_scale rounded to fp16 before the MMA, about 3e-4 relative error), with
 * its device scratch (packed codes, packed scales, pre-scaled activations)
 * taken from one array compiled into the library -- 32 MiB on every GPU that
 * loads it, held until the process exits.
 *
 *   - A, B, a_scale, b_scale and Cf must be device memory on the current CUDA
 *     device (A and Cf 16-byte aligned); nothing is copied.
 *   - A call needing more than the 32 MiB array (about N*K/2 + 2*M*K bytes)
 *     returns ROCKET_E_NOMEM and does nothing.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  The call
 *     is synchronous: it waits for the stream and reads the kernel's status
 *     word before it returns.
 *   - The first call on a device looks up the array's device address (a
 *     one-time set-up on that device); make that first call before any
 *     stream capture.
 *   - Every call on a device shares the one array, so calls that may overlap
 *     on the GPU (other streams, other host threads) race: serialise them. */
int rocket_b200_matmul_int4_groupwise_noalloc(int M, int K, int N, const int8_t *A,
                                              const int8_t *B, const float *a_scale,
                                              const float *b_scale, float *Cf, int group,
                                              void *stream);

/* Group-wise matmul mode for this process (rocket_matmul_int8_groupwise,
 * rocket_matmul_int4_groupwise and the resident _gw entries).
 *   0  precise (default): the reference's definition -- exact integer partial
 *      per K group, scaled by a_scale[m,g] * b_scale[n,g] and summed across
 *      groups in fp32 (src/rocket_matmul.c:2842-2856 of the reference); about
 *      1e-7 relative to the fp64 value, inside its gates' 1e-5 * rms bound.
 *   1  fast: w * b_scale (and a * a_scale when it varies with g) rounded to
 *      fp16 once before an fp16 MMA; about 3e-4 relative Frobenius error.
 * The environment variable ROCKET_GW_FAST=1 selects mode 1 until this is
 * called.  No counterpart in the reference, which has only the first.
 * Returns 0, or ROCKET_E_SHAPE for another value. */
int rocket_b200_gw_mode(int mode);

/* Batched encoder block: nb independent sequences of T tokens stacked along
 * rows (x and out are [nb*T, d]); every projection runs once over all nb*T
 * rows and attention stays within each sequence.  Same arguments and result
 * as nb calls of rocket_encoder_block_fp16 (include/rocket_encoder.h).  No
 * counterpart in the reference, whose API has no batch dimension. */
int rocket_b200_encoder_block_batched_fp16(int fd, int nb, int T, int d, int n_head, int d_ff,
                                           const void *x,
                                           const void *ln1_g, const void *ln1_b,
                                           const void *Wq, const void *bq,
                                           const void *Wk, const void *bk,
                                           const void *Wv, const void *bv,
                                           const void *Wo, const void *bo,
                                           const void *ln2_g, const void *ln2_b,
                                           const void *Wf1, const void *bf1,
                                           const void *Wf2, const void *bf2,
                                           float eps, void *out);

/* Dense GEMM kernel policy for this process (default: automatic).
 *   variant   0 automatic; 128 / 256 single-CTA tiles 128 x 128 / 128 x 256;
 *             384 / 512 CTA-pair tiles 256 x 128 / 256 x 256
 *   stream_k  -1 automatic; 0 never; 1 whenever the pair tiling leaves the last
 *             wave under 90% full (int8 GEMMs only: their int32 sums are exact
 *             in any order)
 * Returns 0, or ROCKET_E_SHAPE for a value outside these. */
int rocket_b200_gemm_policy(int variant, int stream_k);

#ifdef __cplusplus
}
#endif
#endif /* ROCKET_B200_H */
