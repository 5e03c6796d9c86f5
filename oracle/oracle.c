/*
 * oracle.c -- CPU restatement of the reference's host computations for the
 * matmul hot path of librocketnpu (gregordinary/rocket-userspace).
 *
 * TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load this as the checker and the timed CPU baseline; the
 * library (rocket-userspace_b200/) never links or calls it.
 *
 * Pinned against the reference's own gates: oracle/Makefile target `pin`
 * compiles the reference's test programs unchanged against ref_stub.c, whose
 * matmul entry points return this oracle's results; each gate then checks
 * them with its own host loop, its own seeded inputs and its own tolerance
 * (tests/golden/make_golden.py runs them and writes the fixtures).
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

/* ---- fp16 conversion (IEEE binary16, round to nearest even via _Float16) -- */
float orc_h2f(uint16_t h)
{
    _Float16 f;
    memcpy(&f, &h, 2);
    return (float)f;
}

uint16_t orc_f2h(float x)
{
    _Float16 f = (_Float16)x;
    uint16_t h;
    memcpy(&h, &f, 2);
    return h;
}

/* ---- generators ------------------------------------------------------------ */
/* splitmix64 as in tests/matmul_correctness_matrix_rocket.c:50-56 */
uint64_t orc_splitmix64(uint64_t *s)
{
    uint64_t z = (*s += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* glibc rand() stream, e.g. rand()%256-128 (tests/matmul_int8_tiled_rocket.c:36,60) */
void orc_glibc_i8(unsigned seed, int lo, int span, size_t n, int8_t *out)
{
    srand(seed);
    for (size_t i = 0; i < n; i++) out[i] = (int8_t)(rand() % span + lo);
}

void orc_uniform_i8(uint64_t seed, int lo, int hi, size_t n, int8_t *out)
{
    uint64_t s = seed;
    const uint64_t span = (uint64_t)(hi - lo + 1);
    for (size_t i = 0; i < n; i++) out[i] = (int8_t)(lo + (int)(orc_splitmix64(&s) % span));
}

static double u01(uint64_t *s) { return (double)(orc_splitmix64(s) >> 11) * (1.0 / 9007199254740992.0); }

void orc_uniform_f32(uint64_t seed, float lo, float hi, size_t n, float *out)
{
    uint64_t s = seed;
    for (size_t i = 0; i < n; i++) out[i] = (float)(lo + (hi - lo) * u01(&s));
}

/* Box-Muller normals */
static double normal(uint64_t *s, int *have, double *spare)
{
    if (*have) { *have = 0; return *spare; }
    double u1 = u01(s), u2 = u01(s);
    if (u1 < 1e-300) u1 = 1e-300;
    double r = sqrt(-2.0 * log(u1)), th = 2.0 * M_PI * u2;
    *spare = r * sin(th);
    *have = 1;
    return r * cos(th);
}

void orc_normal_f16(uint64_t seed, float scale, size_t n, uint16_t *out)
{
    uint64_t s = seed;
    int have = 0;
    double spare = 0;
    for (size_t i = 0; i < n; i++) out[i] = orc_f2h((float)(normal(&s, &have, &spare) * scale));
}

void orc_normal_f32(uint64_t seed, float mean, float std, size_t n, float *out)
{
    uint64_t s = seed;
    int have = 0;
    double spare = 0;
    for (size_t i = 0; i < n; i++) out[i] = (float)(mean + std * normal(&s, &have, &spare));
}

/* ---- row-range threading --------------------------------------------------- */
typedef struct {
    void (*fn)(void *, int, int);
    void *arg;
    int r0, r1;
} rows_job;

static void *rows_thread(void *p)
{
    rows_job *j = p;
    j->fn(j->arg, j->r0, j->r1);
    return NULL;
}

static void run_rows(void (*fn)(void *, int, int), void *arg, int row0, int row1, int nthreads)
{
    if (nthreads <= 1 || row1 - row0 < 2) { fn(arg, row0, row1); return; }
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    rows_job jb[256];
    int rows = row1 - row0, per = (rows + nthreads - 1) / nthreads, nt = 0;
    for (int t = 0; t < nthreads; t++) {
        int a = row0 + t * per, b = a + per < row1 ? a + per : row1;
        if (a >= b) break;
        jb[t] = (rows_job){fn, arg, a, b};
        if (pthread_create(&th[t], NULL, rows_thread, &jb[t]) != 0) { fn(arg, a, b); jb[t].fn = NULL; }
        nt = t + 1;
    }
    for (int t = 0; t < nt; t++)
        if (jb[t].fn) pthread_join(th[t], NULL);
}

/* ---- int8 x int8 -> int32 via int64 accumulation ----------------------------
 * tests/matmul_int8_tiled_rocket.c:77-83 and tests/matmul_int8_rocket.c:60-69:
 *   s = sum_k (int32)A[m,k] * (int32)B[n,k]  (int64), C = (int32)s            */
typedef struct { int M, K, N; const int8_t *A, *B; int32_t *C; } i8_args;

static void i8_rows(void *p, int r0, int r1)
{
    const i8_args *a = p;
    for (int m = r0; m < r1; m++)
        for (int n = 0; n < a->N; n++) {
            const int8_t *x = a->A + (size_t)m * a->K, *y = a->B + (size_t)n * a->K;
            int64_t s = 0;
            for (int k = 0; k < a->K; k++) s += (int32_t)x[k] * (int32_t)y[k];
            a->C[(size_t)m * a->N + n] = (int32_t)s;
        }
}

void orc_matmul_int8(int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C, int row0,
                     int row1, int nthreads)
{
    i8_args a = {M, K, N, A, B, C};
    run_rows(i8_rows, &a, row0, row1 < 0 ? M : row1, nthreads);
}

/* ---- fp16 x fp16, fp32 accumulation in ascending k, fp16 store --------------
 * tests/matmul_tiled_rocket.c:76-82 (R = fp32 sum) and :92 ((_Float16)R)     */
typedef struct { int M, K, N; const uint16_t *A, *B; float *R; uint16_t *C16; } f16_args;

static void f16_rows(void *p, int r0, int r1)
{
    const f16_args *a = p;
    float *rowA = malloc((size_t)a->K * sizeof(float));
    for (int m = r0; m < r1; m++) {
        for (int k = 0; k < a->K; k++) rowA[k] = orc_h2f(a->A[(size_t)m * a->K + k]);
        for (int n = 0; n < a->N; n++) {
            const uint16_t *y = a->B + (size_t)n * a->K;
            float s = 0.f;
            for (int k = 0; k < a->K; k++) s += rowA[k] * orc_h2f(y[k]);
            if (a->R) a->R[(size_t)m * a->N + n] = s;
            if (a->C16) a->C16[(size_t)m * a->N + n] = orc_f2h(s);
        }
    }
    free(rowA);
}

void orc_matmul_fp16(int M, int K, int N, const uint16_t *A, const uint16_t *B, float *R,
                     uint16_t *C16, int row0, int row1, int nthreads)
{
    f16_args a = {M, K, N, A, B, R, C16};
    run_rows(f16_rows, &a, row0, row1 < 0 ? M : row1, nthreads);
}

/* ---- group-wise: fp64 reference -------------------------------------------------
 * tests/matmul_int8_groupwise_rocket.c:41-56 (ref_gw), also
 * tests/matmul_int4_prepacked_gw_rocket.c:33-47:
 *   ref[m,n] = sum_g (double)as[m,g] * (double)bs[n,g] * (double)ip_g,
 *   ip_g = sum_{k in g} (long)A * (long)B                                         */
typedef struct { int M, K, N, group; const int8_t *A, *B; const float *as, *bs; double *ref; } gw_args;

static void gw_rows(void *p, int r0, int r1)
{
    const gw_args *a = p;
    const int nG = a->K / a->group;
    for (int m = r0; m < r1; m++)
        for (int n = 0; n < a->N; n++) {
            double acc = 0.0;
            for (int g = 0; g < nG; g++) {
                long ip = 0;
                const int8_t *x = a->A + (size_t)m * a->K + (size_t)g * a->group;
                const int8_t *y = a->B + (size_t)n * a->K + (size_t)g * a->group;
                for (int k = 0; k < a->group; k++) ip += (long)x[k] * (long)y[k];
                acc += (double)a->as[(size_t)m * nG + g] * (double)a->bs[(size_t)n * nG + g] * (double)ip;
            }
            a->ref[(size_t)m * a->N + n] = acc;
        }
}

void orc_gw_ref(int M, int K, int N, int group, const int8_t *A, const int8_t *B, const float *as,
                const float *bs, double *ref, int row0, int row1, int nthreads)
{
    gw_args a = {M, K, N, group, A, B, as, bs, ref};
    run_rows(gw_rows, &a, row0, row1 < 0 ? M : row1, nthreads);
}

/* ---- group-wise: the reference library's own fp32 host accumulation ------------
 * src/rocket_matmul.c:2846-2856 / src/rocket_prepacked_int8.c:620-632: for each
 * K-group g in ascending order, Cf += as[m,g] * bs[n,g] * (float)partial_g, in
 * fp32 and in that evaluation order ((as*bs)*partial).  With the K-tile equal
 * to the group this is the value the NPU path returns.                        */
void orc_gw_f32(int M, int K, int N, int group, const int8_t *A, const int8_t *B, const float *as,
                const float *bs, float *Cf)
{
    const int nG = K / group;
    for (size_t i = 0; i < (size_t)M * N; i++) Cf[i] = 0.f;
    for (int g = 0; g < nG; g++)
        for (int m = 0; m < M; m++)
            for (int n = 0; n < N; n++) {
                int32_t p = 0;
                const int8_t *x = A + (size_t)m * K + (size_t)g * group;
                const int8_t *y = B + (size_t)n * K + (size_t)g * group;
                for (int k = 0; k < group; k++) p += (int32_t)x[k] * (int32_t)y[k];
                Cf[(size_t)m * N + n] += as[(size_t)m * nG + g] * bs[(size_t)n * nG + g] * (float)p;
            }
}

/* =========================================================================
 * Encoder ops: fp64 host definitions, fp16 in / fp16 out.  Each restates the
 * reference's public host reference named beside it (pinned against those
 * functions themselves by tests/test_oracle_encoder_pin.py).
 * ========================================================================= */
static double hd(uint16_t h) { return (double)orc_h2f(h); }
static uint16_t dh16(double v)
{
    _Float16 f = (_Float16)v;   /* one rounding, double -> half, as the reference stores */
    uint16_t h;
    memcpy(&h, &f, 2);
    return h;
}

/* src/rocket_norm.c:132-150 (rocket_layernorm_ref_fp16): E[x^2]-mean^2 variance, clamped at 0 */
void orc_layernorm_f16(int M, int H, const uint16_t *x, const uint16_t *g, const uint16_t *b,
                       float eps, uint16_t *y)
{
    for (int m = 0; m < M; m++) {
        const uint16_t *r = x + (size_t)m * H;
        double s1 = 0, s2 = 0;
        for (int i = 0; i < H; i++) { double v = hd(r[i]); s1 += v; s2 += v * v; }
        double mean = s1 / H, var = s2 / H - mean * mean;
        if (var < 0) var = 0;
        double inv = 1.0 / sqrt(var + (double)eps);
        for (int i = 0; i < H; i++)
            y[(size_t)m * H + i] = dh16((hd(r[i]) - mean) * inv * hd(g[i]) + (b ? hd(b[i]) : 0.0));
    }
}

/* src/rocket_norm.c:57-70 (rocket_rmsnorm_ref_fp16) */
void orc_rmsnorm_f16(int M, int H, const uint16_t *x, const uint16_t *w, float eps, uint16_t *y)
{
    for (int m = 0; m < M; m++) {
        const uint16_t *r = x + (size_t)m * H;
        double s2 = 0;
        for (int i = 0; i < H; i++) s2 += hd(r[i]) * hd(r[i]);
        double inv = 1.0 / sqrt(s2 / H + (double)eps);
        for (int i = 0; i < H; i++) y[(size_t)m * H + i] = dh16(hd(r[i]) * inv * hd(w[i]));
    }
}

/* src/rocket_softmax.c:23-35 and :80-92 (softmax / log-softmax, row max shift) */
void orc_softmax_f16(int M, int N, const uint16_t *x, int log_mode, uint16_t *y)
{
    for (int m = 0; m < M; m++) {
        const uint16_t *r = x + (size_t)m * N;
        double mx = -INFINITY, s = 0;
        for (int i = 0; i < N; i++) if (hd(r[i]) > mx) mx = hd(r[i]);
        for (int i = 0; i < N; i++) s += exp(hd(r[i]) - mx);
        for (int i = 0; i < N; i++)
            y[(size_t)m * N + i] = dh16(log_mode ? hd(r[i]) - (mx + log(s)) : exp(hd(r[i]) - mx) / s);
    }
}

/* src/rocket_activation.c:48-77 (act_eval) */
double orc_act(int kind, double x)
{
    double hs = x / 6.0 + 0.5;
    hs = hs < 0 ? 0 : (hs > 1 ? 1 : hs);
    double sp = x > 0 ? x + log1p(exp(-x)) : log1p(exp(x));
    switch (kind) {
    case 0: return 1.0 / (1.0 + exp(-x));
    case 1: return hs;
    case 2: return x * hs;
    case 3: return x * (1.0 / (1.0 + exp(-x)));
    case 4: return tanh(x);
    case 5: return 0.5 * x * (1.0 + erf(x / 1.4142135623730951));
    case 7: return x > 0 ? sqrt(x) : 0;
    case 8: return x > 0 ? 1.0 / sqrt(x) : 0;
    case 9: return x != 0 ? 1.0 / x : 0;
    case 10: return exp(x);
    case 11: return 0.5 * (1.0 + erf(x / 1.4142135623730951));
    case 12: return sp;
    case 13: return tanh(sp);
    case 14: return x * tanh(sp);
    case 15: return fabs(x);
    case 18: return x > 0 ? log(x) : 0;
    default: return 0;
    }
}

void orc_activation_f16(int kind, const uint16_t *x, uint16_t *y, size_t n)
{
    for (size_t i = 0; i < n; i++) y[i] = dh16(orc_act(kind, hd(x[i])));
}

/* the FFN / encoder MLP activation (src/rocket_ffn.c:23-27, src/rocket_encoder.c:22):
 * GELU as 0.5 x (1 + erf(x / sqrt 2)) written with M_SQRT1_2, SiLU as x / (1 + e^-x) */
static double act_mlp(int kind, double g)
{
    if (kind == 5) return 0.5 * g * (1.0 + erf(g * M_SQRT1_2));
    return g / (1.0 + exp(-g));
}

/* y[T, N] = x[T, K] W[N, K]^T (+ b), fp64 */
static void lin64(int T, int K, int N, const double *x, const uint16_t *W, const uint16_t *b, double *y)
{
    for (int t = 0; t < T; t++)
        for (int n = 0; n < N; n++) {
            double a = 0;
            const uint16_t *w = W + (size_t)n * K;
            for (int k = 0; k < K; k++) a += x[(size_t)t * K + k] * hd(w[k]);
            y[(size_t)t * N + n] = a + (b ? hd(b[n]) : 0.0);
        }
}

/* src/rocket_attn.c:41-84 (rocket_mha_self_ref_fp16): q/k/v projections, per-head
 * softmax(q k^T / sqrt(dh)) v in fp64, output projection; one fp16 rounding */
void orc_mha_self_f16(int T, int d, int nh, const uint16_t *x, const uint16_t *Wq, const uint16_t *bq,
                      const uint16_t *Wk, const uint16_t *bk, const uint16_t *Wv, const uint16_t *bv,
                      const uint16_t *Wo, const uint16_t *bo, uint16_t *out)
{
    const int dhd = d / nh;
    const size_t Td = (size_t)T * d;
    double *xd = malloc(Td * sizeof(double)), *q = malloc(Td * sizeof(double));
    double *k = malloc(Td * sizeof(double)), *v = malloc(Td * sizeof(double));
    double *ctx = malloc(Td * sizeof(double)), *p = malloc((size_t)T * sizeof(double));
    double *o = malloc(Td * sizeof(double));
    for (size_t i = 0; i < Td; i++) xd[i] = hd(x[i]);
    lin64(T, d, d, xd, Wq, bq, q);
    lin64(T, d, d, xd, Wk, bk, k);
    lin64(T, d, d, xd, Wv, bv, v);
    const double sc = 1.0 / sqrt((double)dhd);
    for (int h = 0; h < nh; h++)
        for (int i = 0; i < T; i++) {
            double mx = -INFINITY, sum = 0;
            for (int j = 0; j < T; j++) {
                double s = 0;
                for (int c = 0; c < dhd; c++) s += q[(size_t)i * d + h * dhd + c] * k[(size_t)j * d + h * dhd + c];
                p[j] = s * sc;
                if (p[j] > mx) mx = p[j];
            }
            for (int j = 0; j < T; j++) { p[j] = exp(p[j] - mx); sum += p[j]; }
            for (int c = 0; c < dhd; c++) {
                double a = 0;
                for (int j = 0; j < T; j++) a += p[j] * v[(size_t)j * d + h * dhd + c];
                ctx[(size_t)i * d + h * dhd + c] = a / sum;
            }
        }
    lin64(T, d, d, ctx, Wo, bo, o);
    for (size_t i = 0; i < Td; i++) out[i] = dh16(o[i]);
    free(xd); free(q); free(k); free(v); free(ctx); free(p); free(o);
}

/* src/rocket_ffn.c:58-82 (rocket_ffn_ref_fp16): act(x Wg^T) * (x Wu^T), then Wd, fp64 */
void orc_ffn_f16(int M, int H, int I, const uint16_t *x, const uint16_t *Wg, const uint16_t *Wu,
                 const uint16_t *Wd, int kind, uint16_t *out)
{
    double *xd = malloc((size_t)M * H * sizeof(double)), *g = malloc((size_t)M * I * sizeof(double));
    double *u = malloc((size_t)M * I * sizeof(double)), *o = malloc((size_t)M * H * sizeof(double));
    for (size_t i = 0; i < (size_t)M * H; i++) xd[i] = hd(x[i]);
    lin64(M, H, I, xd, Wg, NULL, g);
    lin64(M, H, I, xd, Wu, NULL, u);
    for (size_t i = 0; i < (size_t)M * I; i++) g[i] = act_mlp(kind, g[i]) * u[i];
    lin64(M, I, H, g, Wd, NULL, o);
    for (size_t i = 0; i < (size_t)M * H; i++) out[i] = dh16(o[i]);
    free(xd); free(g); free(u); free(o);
}

/* src/rocket_encoder.c:79-108 (rocket_encoder_block_ref_fp16): pre-norm block;
 * the attention half rounds to fp16 where the reference does (LN output, MHA
 * output, residual sum), the MLP half stays fp64 until the final store */
void orc_encoder_block_f16(int T, int d, int nh, int dff, const uint16_t *x,
                           const uint16_t *g1, const uint16_t *b1, const uint16_t *Wq,
                           const uint16_t *bq, const uint16_t *Wk, const uint16_t *bk,
                           const uint16_t *Wv, const uint16_t *bv, const uint16_t *Wo,
                           const uint16_t *bo, const uint16_t *g2, const uint16_t *b2,
                           const uint16_t *W1, const uint16_t *c1, const uint16_t *W2,
                           const uint16_t *c2, float eps, uint16_t *out)
{
    const size_t Td = (size_t)T * d;
    uint16_t *ln = malloc(Td * 2), *attn = malloc(Td * 2), *xa = malloc(Td * 2);
    double *lnd = malloc(Td * sizeof(double)), *f1 = malloc((size_t)T * dff * sizeof(double));
    double *f2 = malloc(Td * sizeof(double));
    orc_layernorm_f16(T, d, x, g1, b1, eps, ln);
    orc_mha_self_f16(T, d, nh, ln, Wq, bq, Wk, bk, Wv, bv, Wo, bo, attn);
    for (size_t i = 0; i < Td; i++) xa[i] = dh16(hd(x[i]) + hd(attn[i]));
    orc_layernorm_f16(T, d, xa, g2, b2, eps, ln);
    for (size_t i = 0; i < Td; i++) lnd[i] = hd(ln[i]);
    lin64(T, d, dff, lnd, W1, c1, f1);
    for (size_t i = 0; i < (size_t)T * dff; i++) f1[i] = act_mlp(5, f1[i]);
    lin64(T, dff, d, f1, W2, NULL, f2);
    for (size_t i = 0; i < Td; i++) out[i] = dh16(hd(xa[i]) + f2[i] + (c2 ? hd(c2[i % d]) : 0.0));
    free(ln); free(attn); free(xa); free(lnd); free(f1); free(f2);
}

/* ---- reductions (each a double-accumulating row loop) ---- */

/* src/rocket_reduce.c:380-390: out[m] = sum_h in[m, h] (x 1/H when mean) */
void orc_reduce_feature_f16(int M, int H, const uint16_t *x, int mean, float *out)
{
    const double inv = mean ? 1.0 / (double)H : 1.0;
    for (int m = 0; m < M; m++) {
        double acc = 0;
        for (int h = 0; h < H; h++) acc += hd(x[(size_t)m * H + h]);
        out[m] = (float)(acc * inv);
    }
}

/* src/rocket_reduce.c:445-462: inclusive / exclusive, forward / reverse prefix sums */
void orc_cumsum_f16(int M, int N, const uint16_t *x, int exclusive, int reverse, uint16_t *y)
{
    for (int m = 0; m < M; m++) {
        const uint16_t *r = x + (size_t)m * N;
        uint16_t *o = y + (size_t)m * N;
        double acc = 0;
        for (int i = 0; i < N; i++) {
            const int j = reverse ? N - 1 - i : i;
            if (exclusive) { o[j] = dh16(acc); acc += hd(r[j]); }
            else           { acc += hd(r[j]); o[j] = dh16(acc); }
        }
    }
}

/* src/rocket_norm.c:21-30: out[m, n] = (fp16)((float)in[m, n] * r[m]) in float */
void orc_scale_rows_f16(int M, int N, const uint16_t *x, const float *r, uint16_t *y)
{
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++)
            y[(size_t)m * N + n] = dh16((double)(orc_h2f(x[(size_t)m * N + n]) * r[m]));
}

/* src/rocket_softmax.c:141-156: loss = logsumexp(row) - row[target]; out-of-range target -> 0 */
void orc_cross_entropy_f16(int M, int N, const uint16_t *x, const int *target, float *loss)
{
    for (int m = 0; m < M; m++) {
        const uint16_t *r = x + (size_t)m * N;
        double mx = -INFINITY, s = 0;
        for (int n = 0; n < N; n++) if (hd(r[n]) > mx) mx = hd(r[n]);
        for (int n = 0; n < N; n++) s += exp(hd(r[n]) - mx);
        const int t = target[m];
        const double g = (t >= 0 && t < N) ? hd(r[t]) : 0.0;
        loss[m] = (float)(mx + log(s) - g);
    }
}

/* src/rocket_attn.c:181-187 (fa_score) and :189-222 (masked GQA attention host loop):
 * fp64 dot products, the score transform in float, fp64 softmax and P.V */
static float fa_score_ref(float qk, float scale, float softcap, float m)
{
    float s = qk * scale;
    if (softcap != 0.0f) s = softcap * tanhf(s / softcap);
    s += m;
    return s < -30000.0f ? -30000.0f : s;
}

typedef struct {
    int T, n_kv, dh, dv, nh, nkvh;
    float scale, softcap;
    const uint16_t *Q, *K, *V, *mask;
    uint16_t *out;
} fa_args;

/* rows r = h * T + t, each computed independently */
static void fa_rows(void *p, int r0, int r1)
{
    const fa_args *a = p;
    const int T = a->T, n_kv = a->n_kv, dh = a->dh, dv = a->dv, gqa = a->nh / a->nkvh;
    double *sc = malloc((size_t)n_kv * sizeof(double));
    if (!sc) return;
    for (int r = r0; r < r1; r++) {
        const int h = r / T, t = r % T, hk = h / gqa;
        const uint16_t *qr = a->Q + ((size_t)h * T + t) * dh;
        const uint16_t *Kh = a->K + (size_t)hk * n_kv * dh;
        const uint16_t *Vh = a->V + (size_t)hk * dv * n_kv;
        uint16_t *orow = a->out + ((size_t)h * T + t) * dv;
        double mx = -INFINITY;
        for (int j = 0; j < n_kv; j++) {
            double qk = 0;
            for (int c = 0; c < dh; c++) qk += hd(qr[c]) * hd(Kh[(size_t)j * dh + c]);
            const float mj = a->mask ? orc_h2f(a->mask[(size_t)t * n_kv + j]) : 0.0f;
            sc[j] = fa_score_ref((float)qk, a->scale, a->softcap, mj);
            if (sc[j] > mx) mx = sc[j];
        }
        double sum = 0;
        for (int j = 0; j < n_kv; j++) { sc[j] = exp(sc[j] - mx); sum += sc[j]; }
        const double inv = sum > 0 ? 1.0 / sum : 0.0;
        for (int c = 0; c < dv; c++) {
            double acc = 0;
            for (int j = 0; j < n_kv; j++) acc += sc[j] * hd(Vh[(size_t)c * n_kv + j]);
            orow[c] = dh16(acc * inv);
        }
    }
    free(sc);
}

void orc_flash_attn_f16_mt(int T, int n_kv, int dh, int dv, int nh, int nkvh, float scale, float softcap,
                           const uint16_t *Q, const uint16_t *K, const uint16_t *V, const uint16_t *mask,
                           uint16_t *out, int nthreads)
{
    fa_args a = {T, n_kv, dh, dv, nh, nkvh, scale, softcap, Q, K, V, mask, out};
    run_rows(fa_rows, &a, 0, nh * T, nthreads);
}

void orc_flash_attn_f16(int T, int n_kv, int dh, int dv, int nh, int nkvh, float scale, float softcap,
                        const uint16_t *Q, const uint16_t *K, const uint16_t *V, const uint16_t *mask,
                        uint16_t *out)
{
    orc_flash_attn_f16_mt(T, n_kv, dh, dv, nh, nkvh, scale, softcap, Q, K, V, mask, out, 1);
}
