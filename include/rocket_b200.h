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

/* Kernel profiling (the device-side analogue of the reference's
 * ROCKET_MM_PROFILE, src/rocket_matmul.c:74-125).  While enabled (also by the
 * environment variable ROCKET_MM_PROFILE=1), every kernel the library launches
 * is bracketed by CUDA events on its own stream; the elapsed times are
 * accumulated per kernel family when the call completes.  Families are
 * indexed 0..n-1; get returns 0, or ROCKET_E_SHAPE past the last one. */
void  rocket_b200_profile_enable(int on);
void  rocket_b200_profile_reset(void);
int   rocket_b200_profile_get(int idx, const char **name, uint64_t *launches, double *total_ms);

#ifdef __cplusplus
}
#endif
#endif /* ROCKET_B200_H */
