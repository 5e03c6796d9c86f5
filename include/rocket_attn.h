/*
 * rocket_attn.h -- multi-head self-attention, B200 build (reference
 * include/rocket_attn.h:34-43; host definition src/rocket_attn.c:41-84).
 * q/k/v projections on the tcgen05 GEMM (bias fused), one fused attention
 * kernel (scores, online softmax and P.V on the tensor cores, scores never
 * leave the chip), output projection with its bias fused.  head_dim
 * d / n_head must be a multiple of 16 and at most 256 (ROCKET_E_UNSUPPORTED
 * otherwise); 64 runs a kernel holding O in registers, others the flash kernel
 * below.  Biases may be NULL.
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

/* Masked grouped-query attention (reference include/rocket_attn.h:46-150), one
 * fused kernel for all heads.  Per query head h, kv head hk = h / (n_head / n_kv_heads):
 *   S = scale * q_h k_hk^T  [softcap != 0: S = softcap * tanh(S / softcap)]
 *   S = max(S + mask, -30000);  out_h = softmax(S) v_hk
 * Layouts: Q [n_head][n_tokens][head_dim], K [n_kv_heads][n_kv][head_dim],
 * V [n_kv_heads][dv][n_kv], mask [n_tokens][n_kv] additive fp16 or NULL,
 * out [n_head][n_tokens][dv].  head_dim % 32 == 0 and dv % 16 == 0 (reference
 * rules), both <= 256 here.  _mt gives the same result as the single entry;
 * _ctx keeps a device handle across calls. */
typedef struct rocket_fa_ctx rocket_fa_ctx;
rocket_fa_ctx *rocket_fa_ctx_create(int nthreads);
void           rocket_fa_ctx_free(rocket_fa_ctx *c);
int rocket_flash_attn_fp16(int fd, int n_tokens, int n_kv, int head_dim, int dv, int n_head,
                           int n_kv_heads, float scale, float softcap, const _Float16 *Q,
                           const _Float16 *K, const _Float16 *V, const _Float16 *mask, _Float16 *out);
int rocket_flash_attn_fp16_mt(int fd, int n_tokens, int n_kv, int head_dim, int dv, int n_head,
                              int n_kv_heads, float scale, float softcap, const _Float16 *Q,
                              const _Float16 *K, const _Float16 *V, const _Float16 *mask,
                              _Float16 *out, int nthreads);
int rocket_flash_attn_fp16_ctx(rocket_fa_ctx *c, int n_tokens, int n_kv, int head_dim, int dv,
                               int n_head, int n_kv_heads, float scale, float softcap,
                               const _Float16 *Q, const _Float16 *K, const _Float16 *V,
                               const _Float16 *mask, _Float16 *out);
#ifdef __cplusplus
}
#endif
#endif
