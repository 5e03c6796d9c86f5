/*
 * rocket_ffn.h -- gated and plain MLP blocks, B200 build (reference
 * include/rocket_ffn.h:40-98; host definitions src/rocket_ffn.c:23-82).
 * Projections run on the tcgen05 GEMM; bias and GELU / SiLU are fused into
 * the projection's epilogue; the gated product is one element-wise pass.
 * Weights are [out, in] row-major.  `kind` is ROCKET_ACTIVATION_SILU or _GELU.
 */
#ifndef ROCKET_FFN_H
#define ROCKET_FFN_H
#ifdef ROCKET_FLOAT16_T
typedef ROCKET_FLOAT16_T _Float16;
#endif
#ifdef __cplusplus
extern "C" {
#endif
/* prod = act(gate) * up over n elements. */
int rocket_geglu_fp16(int fd, const _Float16 *gate, const _Float16 *up, int kind, _Float16 *prod, int n);
/* out[M,H] = (act(x Wg^T) * (x Wu^T)) Wd^T ; Wg, Wu [I,H], Wd [H,I]. H%32, I%32, M%4. */
int rocket_ffn_fp16(int fd, int M, int H, int I, const _Float16 *x, const _Float16 *Wg,
                    const _Float16 *Wu, const _Float16 *Wd, int kind, _Float16 *out);
int rocket_ffn_fp16_fused(int fd, int M, int H, int I, const _Float16 *x, const _Float16 *Wg,
                          const _Float16 *Wu, const _Float16 *Wd, int kind, _Float16 *out);
/* out[M,Dout] = act(x W1^T + b1) W2^T ; W1 [Dff,Din], b1 [Dff] or NULL, W2 [Dout,Dff].
 * Din%32, Dff%32, Dout%16, M%4. */
int rocket_mlp_fp16_fused(int fd, int M, int Din, int Dff, int Dout, const _Float16 *x,
                          const _Float16 *W1, const _Float16 *b1, const _Float16 *W2, int kind,
                          _Float16 *out);
#ifdef __cplusplus
}
#endif
#endif
