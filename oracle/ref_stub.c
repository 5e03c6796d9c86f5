/*
 * ref_stub.c -- TEST INFRASTRUCTURE ONLY.  A stand-in for the reference's
 * device library, used to pin oracle.c against the reference's own gates.
 *
 * The reference gates (tests/matmul_*_rocket.c of gregordinary/rocket-userspace)
 * are compiled unchanged and linked against this file instead of the NPU
 * library: rocket_open() succeeds, and every matmul entry returns oracle.c's
 * result.  The gate then compares that result with its own host loop on its
 * own seeded inputs under its own tolerance -- so a PASS line means the oracle
 * reproduces the reference's definition.  With ORC_DUMP=<prefix> set, every
 * call also writes its inputs and the oracle's output to <prefix>_<n>.bin
 * (format read by tests/golden/make_golden.py).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

typedef _Float16 f16;

static int g_dump_n;

static void dump(const char *kind, int M, int K, int N, int group, const void *A, size_t asz,
                 const void *B, size_t bsz, const void *as, size_t assz, const void *bs, size_t bssz,
                 const void *C, size_t csz)
{
    const char *pre = getenv("ORC_DUMP");
    if (!pre) return;
    char path[512];
    snprintf(path, sizeof path, "%s_%03d.bin", pre, g_dump_n++);
    FILE *f = fopen(path, "wb");
    if (!f) return;
    char tag[16] = {0};
    strncpy(tag, kind, 15);
    fwrite("RKBG", 1, 4, f);
    fwrite(tag, 1, 16, f);
    int32_t hdr[4] = {M, K, N, group};
    fwrite(hdr, 4, 4, f);
    uint64_t sz[5] = {asz, bsz, assz, bssz, csz};
    fwrite(sz, 8, 5, f);
    if (asz) fwrite(A, 1, asz, f);
    if (bsz) fwrite(B, 1, bsz, f);
    if (assz) fwrite(as, 1, assz, f);
    if (bssz) fwrite(bs, 1, bssz, f);
    if (csz) fwrite(C, 1, csz, f);
    fclose(f);
}

int rocket_open(void) { return 3; }
void rocket_close(int fd) { (void)fd; }

static int plan(int M, int K, int N, int natom, int *Mt, int *Kt, int *Nt)
{
    if (M <= 0 || (M % 4 && M != 1) || K <= 0 || K % 32 || N <= 0 || N % natom) return -1;
    if (Mt) *Mt = M < 256 ? M : 256;
    if (Kt) *Kt = K < 256 ? K : 256;
    if (Nt) *Nt = N < 256 ? N : 256;
    return ((M + 255) / 256) * ((N + 255) / 256) * ((K + 255) / 256);
}
int rocket_matmul_plan(int M, int K, int N, int *Mt, int *Kt, int *Nt) { return plan(M, K, N, 16, Mt, Kt, Nt); }
int rocket_matmul_plan_int8(int M, int K, int N, int *Mt, int *Kt, int *Nt) { return plan(M, K, N, 32, Mt, Kt, Nt); }
int rocket_matmul_plan_int4(int M, int K, int N, int *Mt, int *Kt, int *Nt) { return plan(M, K, N, 64, Mt, Kt, Nt); }
int rocket_matmul_plan_int8_gw(int M, int K, int N, int group, int *Mt, int *Kt, int *Nt)
{
    if (group < 32 || group % 32 || K % group) return -1;
    int r = plan(M, K, N, 32, Mt, Kt, Nt);
    if (r >= 0 && Kt) *Kt = group < 256 ? group : 256;
    return r;
}

int rocket_matmul_int8(int fd, int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C)
{
    (void)fd;
    orc_matmul_int8(M, K, N, A, B, C, 0, M, 1);
    dump("int8", M, K, N, 0, A, (size_t)M * K, B, (size_t)N * K, NULL, 0, NULL, 0, C, (size_t)M * N * 4);
    return 0;
}

int rocket_matmul_int4(int fd, int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C)
{
    (void)fd;
    orc_matmul_int8(M, K, N, A, B, C, 0, M, 1);
    dump("int4", M, K, N, 0, A, (size_t)M * K, B, (size_t)N * K, NULL, 0, NULL, 0, C, (size_t)M * N * 4);
    return 0;
}

int rocket_matmul_fp16(int fd, int M, int K, int N, const f16 *A, const f16 *B, f16 *C)
{
    (void)fd;
    orc_matmul_fp16(M, K, N, (const uint16_t *)A, (const uint16_t *)B, NULL, (uint16_t *)C, 0, M, 1);
    dump("fp16", M, K, N, 0, A, (size_t)M * K * 2, B, (size_t)N * K * 2, NULL, 0, NULL, 0, C,
         (size_t)M * N * 2);
    return 0;
}

int rocket_matmul_fp16_mt(int M, int K, int N, const f16 *A, const f16 *B, f16 *C, int nthreads)
{
    (void)nthreads;
    return rocket_matmul_fp16(0, M, K, N, A, B, C);
}

static int gw(const char *kind, int M, int K, int N, const int8_t *A, const int8_t *B,
              const float *as, const float *bs, float *Cf, int group)
{
    const int nG = K / group;
    double *ref = malloc((size_t)M * N * sizeof(double));
    if (!ref) return -3;
    orc_gw_ref(M, K, N, group, A, B, as, bs, ref, 0, M, 1);
    for (size_t i = 0; i < (size_t)M * N; i++) Cf[i] = (float)ref[i];
    free(ref);
    dump(kind, M, K, N, group, A, (size_t)M * K, B, (size_t)N * K, as, (size_t)M * nG * 4, bs,
         (size_t)N * nG * 4, Cf, (size_t)M * N * 4);
    return 0;
}

int rocket_matmul_int8_groupwise(int fd, int M, int K, int N, const int8_t *A, const int8_t *B,
                                 const float *as, const float *bs, float *Cf, int group)
{
    (void)fd;
    return gw("int8_gw", M, K, N, A, B, as, bs, Cf, group);
}

int rocket_matmul_int4_groupwise(int fd, int M, int K, int N, const int8_t *A, const int8_t *B,
                                 const float *as, const float *bs, float *Cf, int group)
{
    (void)fd;
    return gw("int4_gw", M, K, N, A, B, as, bs, Cf, group);
}

/* resident forms: the "weights" are a host copy of B */
typedef struct { int K, N, group; int8_t *B; } stub_w;
static void *mk_ctx(void) { return calloc(1, 16); }
static stub_w *mk_w(int K, int N, const int8_t *B, int group)
{
    stub_w *w = calloc(1, sizeof *w);
    w->K = K; w->N = N; w->group = group;
    w->B = malloc((size_t)N * K);
    memcpy(w->B, B, (size_t)N * K);
    return w;
}
static void free_w(stub_w *w) { if (w) { free(w->B); free(w); } }

void *rocket_i8_ctx_create(int n) { (void)n; return mk_ctx(); }
void rocket_i8_ctx_free(void *c) { free(c); }
void *rocket_i8_weights_pack(void *c, int M, int K, int N, const int8_t *B) { (void)c; (void)M; return mk_w(K, N, B, 0); }
void *rocket_i8_weights_pack_gw(void *c, int M, int K, int N, const int8_t *B, int g) { (void)c; (void)M; return mk_w(K, N, B, g); }
void rocket_i8_weights_free(void *c, void *w) { (void)c; free_w(w); }
size_t rocket_i8_weights_bytes(const void *w) { const stub_w *s = w; return s ? (size_t)s->N * s->K : 0; }
int rocket_matmul_int8_prepacked(void *c, int M, int K, int N, const int8_t *A, int32_t *C, void *w)
{
    (void)c;
    stub_w *s = w;
    if (K != s->K || N != s->N || M % 4) return -1;
    return rocket_matmul_int8(0, M, K, N, A, s->B, C);
}
int rocket_matmul_int8_prepacked_gw(void *c, int M, int K, int N, const int8_t *A, const float *as,
                                    const float *bs, float *Cf, void *w)
{
    (void)c;
    stub_w *s = w;
    if (K != s->K || N != s->N || M % 4) return -1;
    return gw("int8_gw", M, K, N, A, s->B, as, bs, Cf, s->group);
}

void *rocket_i4_ctx_create(int n) { (void)n; return mk_ctx(); }
void rocket_i4_ctx_free(void *c) { free(c); }
void *rocket_i4_weights_pack(void *c, int M, int K, int N, const int8_t *B) { (void)c; (void)M; return mk_w(K, N, B, 0); }
void *rocket_i4_weights_pack_gw(void *c, int M, int K, int N, const int8_t *B, int g) { (void)c; (void)M; return mk_w(K, N, B, g); }
void rocket_i4_weights_free(void *c, void *w) { (void)c; free_w(w); }
size_t rocket_i4_weights_bytes(const void *w) { const stub_w *s = w; return s ? (size_t)s->N * s->K / 2 : 0; }
int rocket_matmul_int4_prepacked(void *c, int M, int K, int N, const int8_t *A, int32_t *C, void *w)
{
    (void)c;
    stub_w *s = w;
    if (K != s->K || N != s->N || M % 4) return -1;
    return rocket_matmul_int4(0, M, K, N, A, s->B, C);
}
int rocket_matmul_int4_prepacked_gw(void *c, int M, int K, int N, const int8_t *A, const float *as,
                                    const float *bs, float *Cf, void *w)
{
    (void)c;
    stub_w *s = w;
    if (K != s->K || N != s->N || M % 4) return -1;
    return gw("int4_gw", M, K, N, A, s->B, as, bs, Cf, s->group);
}
