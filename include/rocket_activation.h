/*
 * rocket_activation.h -- element-wise activations and binary ops, B200 build
 * (reference include/rocket_activation.h:48-164).  The reference realises
 * these as NPU LUT passes; here each is one fused element-wise kernel with
 * the exact function (CUDA math library) in fp32 on fp16 storage, following
 * the reference's host definitions (src/rocket_activation.c:48-77).
 */
#ifndef ROCKET_ACTIVATION_H
#define ROCKET_ACTIVATION_H
#ifdef ROCKET_FLOAT16_T
typedef ROCKET_FLOAT16_T _Float16;
#endif
#ifdef __cplusplus
extern "C" {
#endif
enum rocket_activation_kind {
    ROCKET_ACTIVATION_SIGMOID     = 0,
    ROCKET_ACTIVATION_HARDSIGMOID = 1,   /* clip(x/6 + 0.5, 0, 1) */
    ROCKET_ACTIVATION_HARDSWISH   = 2,   /* x * hardsigmoid(x) */
    ROCKET_ACTIVATION_SILU        = 3,   /* x * sigmoid(x) */
    ROCKET_ACTIVATION_TANH        = 4,
    ROCKET_ACTIVATION_GELU        = 5,   /* exact erf GELU */
    ROCKET_ACTIVATION_LEAKY_RELU  = 6,   /* parametric: not served by rocket_activation_fp16 */
    ROCKET_ACTIVATION_SQRT        = 7,
    ROCKET_ACTIVATION_RSQRT       = 8,
    ROCKET_ACTIVATION_RECIPROCAL  = 9,
    ROCKET_ACTIVATION_EXP         = 10,
    ROCKET_ACTIVATION_GELU_GATE   = 11,  /* Phi(x) */
    ROCKET_ACTIVATION_SOFTPLUS    = 12,
    ROCKET_ACTIVATION_MISH_GATE   = 13,  /* tanh(softplus(x)) */
    ROCKET_ACTIVATION_MISH        = 14,
    ROCKET_ACTIVATION_ABS         = 15,
    ROCKET_ACTIVATION_ELU         = 16,  /* parametric: not served by rocket_activation_fp16 */
    ROCKET_ACTIVATION_SELU        = 17,  /* parametric: not served by rocket_activation_fp16 */
    ROCKET_ACTIVATION_LOG         = 18,
};
/* out[i] = f(in[i]); ROCKET_E_UNSUPPORTED for the parametric kinds. */
int rocket_activation_fp16(int fd, int kind, const _Float16 *in, _Float16 *out, int n);
int rocket_ew_mul_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n);
int rocket_ew_add_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n);
int rocket_ew_sub_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n);
/* out[i] = max / min(a[i], b[i]) (reference include/rocket_activation.h:170-173) */
int rocket_ew_max_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n);
int rocket_ew_min_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n);
/* out[i] = min(max(in[i], lo), hi) (reference include/rocket_activation.h:178) */
int rocket_clip_fp16(int fd, float lo, float hi, const _Float16 *in, _Float16 *out, int n);
/* "gelu", "silu", ... ; "?" for an unknown kind (reference include/rocket_activation.h:237) */
const char *rocket_activation_name(int kind);
#ifdef __cplusplus
}
#endif
#endif
