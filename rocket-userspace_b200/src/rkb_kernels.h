/*
 * rkb_kernels.h -- internal C ABI between the C host library and the CUDA
 * kernels (the csrc directory).  Plain pointers and sizes only; every function
 * enqueues on the given stream and returns 0 or a negative rocket_status.
 * Pointers are device pointers on the current device.
 */
#ifndef RKB_KERNELS_H
#define RKB_KERNELS_H

#include <stdint.h>
#include <stddef.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

enum rkb_in_kind  { RKB_IN_F16 = 0, RKB_IN_I8 = 1, RKB_IN_BF16 = 2, RKB_IN_TF32 = 3 };
enum rkb_out_kind { RKB_OUT_F16 = 0, RKB_OUT_I32 = 1, RKB_OUT_F32 = 2 };

/* Dense C[M,N] = A[M,K] * B[N,K]^T on tcgen05.  Leading dimensions are in
 * elements; lda/ldb times the element size must be a multiple of 16 bytes and
 * A/B 16-byte aligned (TMA rules), ldc a multiple of 8 and N % 8 == 0.
 * row_scale (length M) / col_scale (length N) are optional fp32 factors
 * applied to each output element in the epilogue (fp16 / fp32 outputs only). */
typedef struct {
    int in_kind, out_kind;
    int M, N, K;
    const void *A; long lda;
    const void *B; long ldb;
    void *C; long ldc;
    const float *row_scale;
    const float *col_scale;
    /* fp16-output epilogue extras (ignored for int32 output):
     *   out = act(acc * row_scale * col_scale + bias[n]) + residual[m * ldr + n] */
    const void *bias;          /* fp16 [N] or NULL */
    int act;                   /* RKB_ACT_* */
    const void *residual;      /* fp16, or NULL */
    long ldr;
    /* workspace sized by rkb_gemm_workspace_bytes: fp32 split-K slabs, or the
     * int8 stream-K tail's sum buffers and counters; may be NULL when that
     * returns 0 (the kernel then runs without either) */
    void *workspace;
} rkb_gemm_desc;

/* Device workspace rkb_gemm_run will use for this descriptor (0 = none). */
size_t rkb_gemm_workspace_bytes(const rkb_gemm_desc *d);
/* kernels one rkb_gemm_run launches (2 with split-K's reduce) */
int rkb_gemm_launches(const rkb_gemm_desc *d);

enum rkb_act { RKB_ACT_NONE = 0, RKB_ACT_GELU = 1, RKB_ACT_SILU = 2 };

int rkb_gemm_run(const rkb_gemm_desc *d, int *err_word, cudaStream_t stream);

/* Group-wise / int4 weight GEMM with in-register dequantisation.
 * Weights are in the resident tiled layout written by rkb_pack_weights:
 * for each 256-row N tile and each 64-wide K block, a contiguous block of
 * 256 x 64 codes (int8: 16 KB, int4: 8 KB nibble-packed) followed in a
 * separate array by 256 x 2 fp16 scales (one per 32-wide K sub-group).
 * A is int8 [M, K] (or fp16 when a_f16 != 0, already scaled per group).
 * Output: fp32 or fp16 [M, N] (ldc), times row_scale[m] when given. */
typedef struct {
    int M, N, K;
    int w_bits;               /* 8 or 4 */
    int a_f16;                /* A is fp16 (pre-scaled) instead of int8 */
    const void *A; long lda;  /* elements */
    const void *Wq;           /* tiled codes */
    const void *Ws;           /* tiled fp16 scales */
    void *C; long ldc; int out_kind;
    const float *row_scale;
    /* exact-partial (precise) group-wise form only, rkb_wgemm_xi_run:
     * A holds the int8 activations (a_f16 == 0), Ws is unused */
    const float *b_scale;     /* fp32 [N, K/group] */
    const float *a_scale_t;   /* fp32 [K/group, M] when a_scale varies with g, else NULL */
    int group;
} rkb_wgemm_desc;

int rkb_wgemm_run(const rkb_wgemm_desc *d, int *err_word, cudaStream_t stream);
/* The a_f16 (group-wise) form with the dequantised weights fed from TMEM;
 * rkb_wgemm_run routes a_f16 descriptors here. */
int rkb_wgemm_ts_run(const rkb_wgemm_desc *d, int *err_word, cudaStream_t stream);

/* Precise group-wise form on the int8 tensor cores: int8 activations as they
 * are (a_f16 == 0, lda in bytes), one exact int32 partial per group, scaled
 * by b_scale[n,g] (x a_scale_t[g,m]) and summed across groups in fp32.
 * row_scale, when given, is applied at the end (a_scale constant along g). */
int rkb_wgemm_xi_run(const rkb_wgemm_desc *d, int *err_word, cudaStream_t stream);
/* a_scale [M, nG] -> [nG, M] */
int rkb_scale_transpose(const float *a_scale, int M, int nG, float *dst, cudaStream_t s);

/* Resident-weight packers (device -> device).  src is the row-major int8
 * weight [N, K] (values in [-8,7] when bits == 4); dst gets the tiled layout
 * above.  N is padded up to the 256-row tile with zero codes.  Returns bytes
 * needed when dst == NULL. */
size_t rkb_wpack_codes_bytes(int N, int K, int bits);
size_t rkb_wpack_scales_bytes(int N, int K);
int rkb_wpack_codes(const int8_t *src, int N, int K, int bits, void *dst, cudaStream_t s);
/* scales: fp32 [N, K/group] -> tiled fp16 [ntile][kblock][256][2]. */
int rkb_wpack_scales(const float *b_scale, int N, int K, int group, void *dst, cudaStream_t s);
/* Unit scales (all 1.0) for the per-channel int4 raw path. */
int rkb_wpack_unit_scales(int N, int K, void *dst, cudaStream_t s);
/* A int8 [M,K] * a_scale[m, k/group] -> fp16 [M,K] (pre-scaled activations). */
int rkb_prescale_a(const int8_t *A, const float *a_scale, int M, int K, int group,
                   void *dst, cudaStream_t s);
/* Rows of a_scale [M, nG] all constant?  Host-side check result is passed in
 * by the caller; this only gathers a_scale[m*nG] into a dense [M] vector. */
int rkb_gather_row_scale(const float *a_scale, int M, int nG, float *dst, cudaStream_t s);

/* ---- encoder ops (csrc/rowops.cu, csrc/attn_tc.cu); fp16 storage ---- */
int rkb_norm_rows(const void *x, const void *gamma, const void *beta, int M, int H, float eps,
                  int rms, void *out, cudaStream_t s);
int rkb_softmax_rows(const void *x, int M, int N, int log_mode, void *out, cudaStream_t s);
/* op: 0 act(a), 1 a+b, 2 a*b, 3 a-b, 4 act(a)*b, 5 max(a,b), 6 min(a,b),
 * 7 clip(a, lo, hi); kind = rocket_activation_kind */
int rkb_elementwise(const void *a, const void *b, int op, int kind, size_t n, void *out,
                    cudaStream_t s);
int rkb_elementwise_ex(const void *a, const void *b, int op, int kind, float lo, float hi, size_t n,
                       void *out, cudaStream_t s);
/* qkv [B*T, 3*H*dh] (row pitch ld) -> Q, K [B*H, Tp, dh], Vt [B*H, dh, Tp], zero padded */
int rkb_split_heads(const void *qkv, long ld, int B, int T, int Tp, int H, int dh, void *Q,
                    void *K, void *Vt, cudaStream_t s);
/* masked GQA flash attention (csrc/fa_tc.cu): Q [nh][T][dh], K [nkvh][n_kv][dh],
 * V [nkvh][dv] rows of ldv elements, mask [T][n_kv] or NULL, out [nh][T][dv] */
int rkb_flash_attn(const void *Q, const void *K, const void *V, long ldv, const void *mask, void *out,
                   int T, int n_kv, int dh, int dv, int n_head, int n_kv_heads, float scale,
                   float softcap, int *err, cudaStream_t stream);
/* general addressing: per-head row counts q_rows / kv_rows in the Q / K arrays;
 * out(h, t) = out + (h / hb) * bstride + (h % hb) * dv + t * ldo */
int rkb_flash_attn_ex(const void *Q, const void *K, const void *V, long ldv, const void *mask, void *out,
                      int T, int n_kv, int dh, int dv, int n_head, int n_kv_heads, float scale,
                      float softcap, int q_rows, int kv_rows, int hb, long bstride, long ldo, int *err,
                      cudaStream_t stream);
/* out[b*T + t, h*dh + c] = softmax(Q K^T * scale) V per (b, h); dh == 64, Tp % 128 == 0 */
int rkb_attention(const void *Q, const void *K, const void *Vt, int B, int H, int T, int Tp,
                  int dh, float scale, void *out, long ldo, int *err, cudaStream_t stream);

int rkb_reduce_rows(const void *x, int M, int H, int mean, float *out, cudaStream_t s);
int rkb_cumsum_rows(const void *x, int M, int N, int exclusive, int reverse, void *out, cudaStream_t s);
int rkb_scale_rows(const void *x, const float *r, int M, int N, void *out, cudaStream_t s);
int rkb_cross_entropy_rows(const void *x, const int *target, int M, int N, float *loss, cudaStream_t s);

/* dst = [a | b | c] (bytes each, 16-byte multiple, aligned device pointers; NULL part -> zeros) */
int rkb_concat3(const void *a, const void *b, const void *c, size_t bytes, void *dst, cudaStream_t s);

/* ---- dtype helpers (csrc/rkb_util.cu) ---- */
int rkb_f32_to_bf16(const void *src, size_t n, void *dst, cudaStream_t s);     /* truncating */
int rkb_int16_split(const int16_t *src, size_t n, int8_t *hi, int8_t *lo, cudaStream_t s);
int rkb_int16_combine(const int32_t *hh, const int32_t *hl, const int32_t *lh, const int32_t *ll,
                      size_t n, int64_t *out, cudaStream_t s);

/* Device properties cached per device. */
int rkb_device_sm_count(int dev);

#ifdef __cplusplus
}
#endif
#endif /* RKB_KERNELS_H */
