/*
 * rocket_softmax.h -- row softmax / log-softmax, B200 build (reference
 * include/rocket_softmax.h; host definitions src/rocket_softmax.c:23-35, :80-92).
 * One warp per row: max, sum of exp, write -- fp32 math on fp16 storage.
 */
#ifndef ROCKET_SOFTMAX_H
#define ROCKET_SOFTMAX_H
#ifdef ROCKET_FLOAT16_T
typedef ROCKET_FLOAT16_T _Float16;
#endif
#ifdef __cplusplus
extern "C" {
#endif
int rocket_softmax_fp16(int fd, int M, int N, const _Float16 *in, _Float16 *out);
int rocket_logsoftmax_fp16(int fd, int M, int N, const _Float16 *in, _Float16 *out);
/* loss[m] = logsumexp(logits[m, :]) - logits[m, target[m]] (fp32 [M]); a target
 * outside [0, N) contributes 0 for the logit term, as in src/rocket_softmax.c:141-155. */
int rocket_cross_entropy_fp16(int fd, int M, int N, const _Float16 *logits, const int *target,
                              float *loss);
#ifdef __cplusplus
}
#endif
#endif
