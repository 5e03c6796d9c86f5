/*
 * rocket_attn.h -- multi-head self-attention, B200 build (reference
 * include/rocket_attn.h:34-43; host definition src/rocket_attn.c:41-84).
 * q/k/v projections on the tcgen05 GEMM (bias fused), one fused attention
 * kernel (scores, online softmax and P.V on the tensor cores, scores never
 * leave the chip), output projection with its bias fused.  head_dim
 * d / n_head must be 64 (ROCKET_E_UNSUPPORTED otherwise).  Biases may be NULL.
 */
#ifndef ROCKET_ATTN_H
#define ROCKET_ATTN_H
#ifdef ROCKET_FLOAT16_T
typedef ROCKET_FLOAT16_T _Float16;
#endif
#ifdef __cplusplus
extern "C" {
#endif
int rocket_mha_self_fp16(int fd, int T, int d, int n_head, const _Float16 *x,
                         const _Float16 *Wq, const _Float16 *bq, const _Float16 *Wk,
                         const _Float16 *bk, const _Float16 *Wv, const _Float16 *bv,
                         const _Float16 *Wo, const _Float16 *bo, _Float16 *out);
#ifdef __cplusplus
}
#endif
#endif
