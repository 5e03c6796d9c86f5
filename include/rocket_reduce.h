/*
 * rocket_reduce.h -- row reductions and prefix sums, B200 build (reference
 * include/rocket_reduce.h:151-199; host definitions src/rocket_reduce.c:380-464).
 * One warp per row, fp32 accumulation.
 */
#ifndef ROCKET_REDUCE_H
#define ROCKET_REDUCE_H
#ifdef ROCKET_FLOAT16_T
typedef ROCKET_FLOAT16_T _Float16;
#endif
#ifdef __cplusplus
extern "C" {
#endif
/* out[m] = sum_h in[m, h] (mean != 0: divided by H), fp32 [M]. */
int rocket_reduce_feature_fp16(int fd, int M, int H, const _Float16 *in, float *out, int mean);
/* per-row prefix sums, fp16 [M, N]; exclusive: skip in[j] at j; reverse: right to left. */
int rocket_cumsum_fp16(int fd, int M, int N, const _Float16 *in, _Float16 *out,
                       int exclusive, int reverse);
#ifdef __cplusplus
}
#endif
#endif
