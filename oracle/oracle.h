/*
 * oracle.h -- CPU restatement of the reference's host computations for the
 * matmul hot path and the encoder ops.  TEST INFRASTRUCTURE ONLY: used by
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the
 * checker / CPU baseline, never by the library.
 */
#ifndef RKB_ORACLE_H
#define RKB_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- generators ---- */
uint64_t orc_splitmix64(uint64_t *state);
/* glibc rand() streams as the reference gates draw them (srand(seed) first). */
void orc_glibc_i8(unsigned seed, int lo, int span, size_t n, int8_t *out);  /* rand()%span + lo */
void orc_uniform_i8(uint64_t seed, int lo, int hi, size_t n, int8_t *out);  /* [lo,hi] */
void orc_uniform_f32(uint64_t seed, float lo, float hi, size_t n, float *out);
void orc_normal_f16(uint64_t seed, float scale, size_t n, uint16_t *out);   /* N(0,1)*scale */
void orc_normal_f32(uint64_t seed, float mean, float std, size_t n, float *out);

/* ---- matmul restatements (C = A * B^T, row-major) ---- */
void orc_matmul_int8(int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C,
                     int row0, int row1, int nthreads);
void orc_matmul_fp16(int M, int K, int N, const uint16_t *A, const uint16_t *B, float *R,
                     uint16_t *C16, int row0, int row1, int nthreads);
void orc_gw_ref(int M, int K, int N, int group, const int8_t *A, const int8_t *B,
                const float *as, const float *bs, double *ref, int row0, int row1, int nthreads);
void orc_gw_f32(int M, int K, int N, int group, const int8_t *A, const int8_t *B,
                const float *as, const float *bs, float *Cf);

/* fp16 helpers */
float    orc_h2f(uint16_t h);
uint16_t orc_f2h(float f);

/* ---- encoder ops (fp64 host definitions; fp16 in / out) ---- */
void orc_layernorm_f16(int M, int H, const uint16_t *x, const uint16_t *g, const uint16_t *b,
                       float eps, uint16_t *y);
void orc_rmsnorm_f16(int M, int H, const uint16_t *x, const uint16_t *w, float eps, uint16_t *y);
void orc_softmax_f16(int M, int N, const uint16_t *x, int log_mode, uint16_t *y);
double orc_act(int kind, double x);
void orc_activation_f16(int kind, const uint16_t *x, uint16_t *y, size_t n);
void orc_mha_self_f16(int T, int d, int nh, const uint16_t *x, const uint16_t *Wq, const uint16_t *bq,
                      const uint16_t *Wk, const uint16_t *bk, const uint16_t *Wv, const uint16_t *bv,
                      const uint16_t *Wo, const uint16_t *bo, uint16_t *out);
void orc_ffn_f16(int M, int H, int I, const uint16_t *x, const uint16_t *Wg, const uint16_t *Wu,
                 const uint16_t *Wd, int kind, uint16_t *out);
void orc_encoder_block_f16(int T, int d, int nh, int dff, const uint16_t *x,
                           const uint16_t *g1, const uint16_t *b1, const uint16_t *Wq,
                           const uint16_t *bq, const uint16_t *Wk, const uint16_t *bk,
                           const uint16_t *Wv, const uint16_t *bv, const uint16_t *Wo,
                           const uint16_t *bo, const uint16_t *g2, const uint16_t *b2,
                           const uint16_t *W1, const uint16_t *c1, const uint16_t *W2,
                           const uint16_t *c2, float eps, uint16_t *out);

/* reductions */
void orc_reduce_feature_f16(int M, int H, const uint16_t *x, int mean, float *out);
void orc_cumsum_f16(int M, int N, const uint16_t *x, int exclusive, int reverse, uint16_t *y);
void orc_scale_rows_f16(int M, int N, const uint16_t *x, const float *r, uint16_t *y);
void orc_cross_entropy_f16(int M, int N, const uint16_t *x, const int *target, float *loss);

/* masked grouped-query attention */
void orc_flash_attn_f16(int T, int n_kv, int dh, int dv, int nh, int nkvh, float scale, float softcap,
                        const uint16_t *Q, const uint16_t *K, const uint16_t *V, const uint16_t *mask,
                        uint16_t *out);
void orc_flash_attn_f16_mt(int T, int n_kv, int dh, int dv, int nh, int nkvh, float scale, float softcap,
                           const uint16_t *Q, const uint16_t *K, const uint16_t *V, const uint16_t *mask,
                           uint16_t *out, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
