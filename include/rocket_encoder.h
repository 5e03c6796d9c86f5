/*
 * rocket_encoder.h -- one pre-norm transformer encoder block, B200 build
 * (reference include/rocket_encoder.h:28-49; host definition
 * src/rocket_encoder.c:79-108):
 *     x = x + MHA(LN1(x));  out = x + GELU(LN2(x) W1^T + b1) W2^T + b2
 * Eight kernels: LN, one fused q/k/v GEMM (N = 3d), head split, fused
 * attention, output projection with bias + residual fused, LN, fc1 with bias
 * + GELU fused, fc2 with bias + residual fused (plus one gather of the q/k/v
 * weights when they are device-resident).  head_dim must be a multiple of 16
 * and at most 256.
 */
#ifndef ROCKET_ENCODER_H
#define ROCKET_ENCODER_H
#ifdef ROCKET_FLOAT16_T
typedef ROCKET_FLOAT16_T _Float16;
#endif
#ifdef __cplusplus
extern "C" {
#endif
int rocket_encoder_block_fp16(int fd, int T, int d, int n_head, int d_ff, const _Float16 *x,
                              const _Float16 *ln1_g, const _Float16 *ln1_b,
                              const _Float16 *Wq, const _Float16 *bq,
                              const _Float16 *Wk, const _Float16 *bk,
                              const _Float16 *Wv, const _Float16 *bv,
                              const _Float16 *Wo, const _Float16 *bo,
                              const _Float16 *ln2_g, const _Float16 *ln2_b,
                              const _Float16 *Wf1, const _Float16 *bf1,
                              const _Float16 *Wf2, const _Float16 *bf2,
                              float eps, _Float16 *out);
#ifdef __cplusplus
}
#endif
#endif
