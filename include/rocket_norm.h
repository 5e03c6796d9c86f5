/*
 * rocket_norm.h -- row normalisations, B200 build (reference include/rocket_norm.h).
 * One warp per row, fp32 statistics over fp16 storage, one pass over HBM.
 * x / out [M, H] row-major fp16; gamma / weight / beta [H] (beta may be NULL).
 * Returns 0 or a negative rocket_status.  The reference's fd < 0 "host
 * reference" mode is not offered: there is no CPU path in this library.
 */
#ifndef ROCKET_NORM_H
#define ROCKET_NORM_H
#ifdef ROCKET_FLOAT16_T
typedef ROCKET_FLOAT16_T _Float16;
#endif
#ifdef __cplusplus
extern "C" {
#endif
/* out[m, n] = in[m, n] * r[m] (r fp32 [M]).  Replaces src/rocket_norm.c:21-60. */
int rocket_scale_rows_fp16(int fd, int M, int N, const _Float16 *in, const float *r, _Float16 *out);
/* out = x / sqrt(mean(x^2) + eps) * weight.  Replaces src/rocket_norm.c:72-126. */
int rocket_rmsnorm_fp16(int fd, int M, int H, const _Float16 *x, const _Float16 *weight,
                        float eps, _Float16 *out);
/* out = (x - mean) / sqrt(var + eps) * gamma + beta.  Replaces src/rocket_norm.c:152-227. */
int rocket_layernorm_fp16(int fd, int M, int H, const _Float16 *x, const _Float16 *gamma,
                          const _Float16 *beta, float eps, _Float16 *out);
#ifdef __cplusplus
}
#endif
#endif
