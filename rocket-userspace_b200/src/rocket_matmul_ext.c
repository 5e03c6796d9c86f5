/*
 * rocket_matmul_ext.c -- the remaining one-shot dtypes and the batched
 * same-shape matmul.
 *
 * Reference: src/rocket_matmul.c (fp16 -> fp32 out :3620, batch :2042-2330,
 * bf16 :3454, tf32 :3840, int16 exact :3377; plans beside each).  On the NPU
 * these are separate register programs (bf16 / tf32 / int16 precision modes);
 * on B200 they are the same tcgen05 GEMM with another operand kind:
 *   bf16   fp32 inputs truncated to bf16 (as the reference's pack does), MMA
 *          kind::f16 with bf16 operands, fp32 accumulate and output
 *   tf32   fp32 inputs fed as-is to MMA kind::tf32, fp32 accumulate and output
 *   int16  each operand split into signed hi / lo bytes (v = 256 hi + lo,
 *          v clamped to [-32768, 32639] like the reference), four exact int8
 *          GEMMs, recombined in int64: 65536 hh + 256 (hl + lh) + ll
 */
#include <stdlib.h>
#include <string.h>

#include "rocket_matmul.h"
#include "rkb_internal.h"

static int m_ok(int M) { return M > 0 && (M % 4 == 0 || M == 1); }

/* int16 / bf16 share the plan geometry (reference include/rocket_matmul.h:487) */
int rocket_matmul_plan_int16(int M, int K, int N, int *Mt, int *Kt, int *Nt)
{
    return rocket_matmul_plan(M, K, N, Mt, Kt, Nt);
}

int rocket_matmul_plan_bf16(int M, int K, int N, int *Mt, int *Kt, int *Nt)
{
    return rocket_matmul_plan_int16(M, K, N, Mt, Kt, Nt);
}

int rocket_matmul_plan_tf32(int M, int K, int N, int *Mt, int *Kt, int *Nt)
{
    if (!m_ok(M) || K <= 0 || N <= 0 || K % 16 || N % 16) return ROCKET_E_SHAPE;
    if (Mt) *Mt = M < 128 ? M : 128;
    if (Kt) *Kt = K < 32 ? K : 32;
    if (Nt) *Nt = N < 256 ? N : 256;
    return ((M + 127) / 128) * ((N + 255) / 256);
}

int rocket_matmul_fp16_f32out(int fd, int M, int K, int N, const _Float16 *A, const _Float16 *B,
                              float *C)
{
    if (rocket_matmul_plan(M, K, N, NULL, NULL, NULL) < 0) return ROCKET_E_SHAPE;
    return rkb_oneshot_dense("rocket_matmul_fp16_f32out", fd, RKB_IN_F16, RKB_OUT_F32, M, K, N, A, B, C, 1);
}

int rocket_matmul_tf32(int fd, int M, int K, int N, const float *A, const float *B, float *C)
{
    if (rocket_matmul_plan_tf32(M, K, N, NULL, NULL, NULL) < 0) return ROCKET_E_SHAPE;
    return rkb_oneshot_dense("rocket_matmul_tf32", fd, RKB_IN_TF32, RKB_OUT_F32, M, K, N, A, B, C, 1);
}

int rocket_matmul_fp16_batch(int fd, int M, int K, int N, int nbatch, const _Float16 *const *A,
                             const _Float16 *const *B, _Float16 *const *C)
{
    const char *who = "rocket_matmul_fp16_batch";
    if (nbatch < 1 || !A || !B || !C || rocket_matmul_plan(M, K, N, NULL, NULL, NULL) < 0 ||
        (M % 4 && nbatch > 1))
        return ROCKET_E_SHAPE;
    if (nbatch == 1) return rocket_matmul_fp16(fd, M, K, N, A[0], B[0], C[0]);
    rkb_handle *h = rkb_get(fd);
    if (!h) return ROCKET_E_DEVICE;
    int rc = 0;
    /* all items queue on the handle's stream; one bounded wait at the end */
    for (int i = 0; i < nbatch && !rc; i++)
        rc = rkb_oneshot_dense(who, fd, RKB_IN_F16, RKB_OUT_F16, M, K, N, A[i], B[i], C[i], 0);
    int fr = rkb_finish(h, who);
    return rc ? rc : fr;
}

struct rocket_mm_batch { int fd; };

rocket_mm_batch *rocket_mm_batch_create(int fd)
{
    if (!rkb_get(fd)) return NULL;
    rocket_mm_batch *b = calloc(1, sizeof *b);
    if (b) b->fd = fd;
    return b;
}

void rocket_mm_batch_free(rocket_mm_batch *b) { free(b); }

int rocket_mm_batch_run(rocket_mm_batch *b, int M, int K, int N, int nbatch, const _Float16 *const *A,
                        const _Float16 *const *B, _Float16 *const *C)
{
    if (!b) return ROCKET_E_SHAPE;
    return rocket_matmul_fp16_batch(b->fd, M, K, N, nbatch, A, B, C);
}

int rocket_matmul_bf16(int fd, int M, int K, int N, const float *A, const float *B, float *C)
{
    const char *who = "rocket_matmul_bf16";
    if (rocket_matmul_plan_bf16(M, K, N, NULL, NULL, NULL) < 0 || !A || !B || !C) return ROCKET_E_SHAPE;
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const size_t na = (size_t)M * K, nb = (size_t)N * K;
    const void *dA = rkb_call_in(&c, A, na * 4);
    const void *dB = rkb_call_in(&c, B, nb * 4);
    void *a16 = rkb_call_tmp(&c, na * 2), *b16 = rkb_call_tmp(&c, nb * 2);
    void *dC = rkb_call_out(&c, C, (size_t)M * N * 4);
    if (!c.rc) {
        rkb_call_check(&c, rkb_f32_to_bf16(dA, na, a16, c.h->stream));
        rkb_call_check(&c, rkb_f32_to_bf16(dB, nb, b16, c.h->stream));
        rkb_count(0, 2);
    }
    rkb_call_gemm_kind(&c, RKB_IN_BF16, RKB_OUT_F32, M, N, K, a16, K, b16, K, dC, N);
    return rkb_call_end(&c);
}

int rocket_matmul_int16_exact(int fd, int M, int K, int N, const int16_t *A, const int16_t *B, int64_t *C)
{
    const char *who = "rocket_matmul_int16_exact";
    if (!m_ok(M) || K <= 0 || N <= 0 || K % 32 || N % 32 || !A || !B || !C) return ROCKET_E_SHAPE;
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const size_t na = (size_t)M * K, nb = (size_t)N * K, nc = (size_t)M * N;
    const int16_t *dA = rkb_call_in(&c, A, na * 2);
    const int16_t *dB = rkb_call_in(&c, B, nb * 2);
    int8_t *ah = rkb_call_tmp(&c, na), *al = rkb_call_tmp(&c, na);
    int8_t *bh = rkb_call_tmp(&c, nb), *bl = rkb_call_tmp(&c, nb);
    int32_t *p[4];
    for (int i = 0; i < 4; i++) p[i] = rkb_call_tmp(&c, nc * 4);
    int64_t *dC = rkb_call_out(&c, C, nc * 8);
    if (!c.rc) {
        rkb_call_check(&c, rkb_int16_split(dA, na, ah, al, c.h->stream));
        rkb_call_check(&c, rkb_int16_split(dB, nb, bh, bl, c.h->stream));
        rkb_count(0, 3);
    }
    rkb_call_gemm_kind(&c, RKB_IN_I8, RKB_OUT_I32, M, N, K, ah, K, bh, K, p[0], N);
    rkb_call_gemm_kind(&c, RKB_IN_I8, RKB_OUT_I32, M, N, K, ah, K, bl, K, p[1], N);
    rkb_call_gemm_kind(&c, RKB_IN_I8, RKB_OUT_I32, M, N, K, al, K, bh, K, p[2], N);
    rkb_call_gemm_kind(&c, RKB_IN_I8, RKB_OUT_I32, M, N, K, al, K, bl, K, p[3], N);
    if (!c.rc) rkb_call_check(&c, rkb_int16_combine(p[0], p[1], p[2], p[3], nc, dC, c.h->stream));
    return rkb_call_end(&c);
}
