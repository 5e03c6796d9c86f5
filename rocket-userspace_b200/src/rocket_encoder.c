/*
 * rocket_encoder.c -- the encoder ops on top of the matmul path: norms,
 * softmax, activations / element-wise ops, gated FFN, MLP, multi-head
 * self-attention and the pre-norm encoder block.
 *
 * Reference: src/rocket_norm.c, src/rocket_softmax.c, src/rocket_activation.c,
 * src/rocket_ffn.c, src/rocket_attn.c:92-176, src/rocket_encoder.c:117-192.
 * There every op is assembled from NPU matmuls, LUT passes, element-wise
 * passes and ones-matmul reductions with host glue between them.  Here each op
 * is a short sequence of kernel launches on the handle's stream with fusion
 * where a pass can be saved: bias / activation / residual ride in the GEMM
 * epilogue, attention is one fused kernel.  Temporaries come from CUDA's
 * stream-ordered allocator (pooled after the first call).  Every entry is
 * synchronous and returns 0 or a negative rocket_status; fd < 0 is an error
 * (the reference's host-reference mode is not offered -- no CPU path).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "rocket_activation.h"
#include "rocket_attn.h"
#include "rocket_b200.h"
#include "rocket_encoder.h"
#include "rocket_ffn.h"
#include "rocket_norm.h"
#include "rocket_softmax.h"
#include "rkb_internal.h"

#define ENC_MAX_TMP 48

typedef struct {
    rkb_handle *h;
    const char *who;
    void *tmp[ENC_MAX_TMP];
    int ntmp;
    int rc;
    struct { void *user; const void *dev; size_t bytes; } outs[4];
    int nouts;
} enc_call;

static int enc_begin(enc_call *c, int fd, const char *who)
{
    memset(c, 0, sizeof *c);
    c->who = who;
    c->h = rkb_get(fd);
    if (!c->h) {
        ROCKET_LOGE("%s: bad device handle %d\n", who, fd);
        return ROCKET_E_DEVICE;
    }
    static int pool_ready[64];
    int dev = c->h->device;
    if (dev < 64 && !pool_ready[dev]) {
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
            uint64_t thr = UINT64_MAX;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
        }
        cudaGetLastError();
        pool_ready[dev] = 1;
    }
    return 0;
}

static void *enc_tmp(enc_call *c, size_t bytes)
{
    if (c->rc || c->ntmp >= ENC_MAX_TMP) { if (!c->rc) c->rc = ROCKET_E_NOMEM; return NULL; }
    void *p = NULL;
    if (cudaMallocAsync(&p, bytes ? bytes : 16, c->h->stream) != cudaSuccess) {
        cudaGetLastError();
        c->rc = ROCKET_E_NOMEM;
        return NULL;
    }
    c->tmp[c->ntmp++] = p;
    return p;
}

/* device view of a caller input (NULL stays NULL) */
static const void *enc_in(enc_call *c, const void *user, size_t bytes)
{
    if (!user || c->rc) return NULL;
    if (rkb_ptr_device(user) == c->h->device && ((uintptr_t)user & 15) == 0) return user;
    void *d = enc_tmp(c, bytes);
    if (d && cudaMemcpyAsync(d, user, bytes, cudaMemcpyDefault, c->h->stream) != cudaSuccess) {
        cudaGetLastError();
        c->rc = ROCKET_E_DEVICE;
    }
    return d;
}

/* device buffer for a caller output; copied back in enc_end when needed */
static void *enc_out(enc_call *c, void *user, size_t bytes)
{
    if (c->rc) return NULL;
    if (rkb_ptr_device(user) == c->h->device && ((uintptr_t)user & 15) == 0) return user;
    void *d = enc_tmp(c, bytes);
    if (d && c->nouts < 4) {
        c->outs[c->nouts].user = user;
        c->outs[c->nouts].dev = d;
        c->outs[c->nouts].bytes = bytes;
        c->nouts++;
    }
    return d;
}

static void enc_check(enc_call *c, int rc)
{
    if (!c->rc && rc) c->rc = rc;
}

static int enc_end(enc_call *c)
{
    for (int i = 0; i < c->nouts && !c->rc; i++)
        if (cudaMemcpyAsync(c->outs[i].user, c->outs[i].dev, c->outs[i].bytes, cudaMemcpyDefault,
                            c->h->stream) != cudaSuccess) {
            cudaGetLastError();
            c->rc = ROCKET_E_DEVICE;
        }
    for (int i = 0; i < c->ntmp; i++) cudaFreeAsync(c->tmp[i], c->h->stream);
    rkb_count(1, 0);
    int fr = rkb_finish(c->h, c->who);
    return c->rc ? c->rc : fr;
}

/* GEMM with fp16 output and fused epilogue: C = act(A W^T + bias) + residual */
static void enc_gemm(enc_call *c, int M, int N, int K, const void *A, long lda, const void *W,
                     void *C, long ldc, const void *bias, int act, const void *res, long ldr)
{
    if (c->rc) return;
    rkb_gemm_desc d;
    memset(&d, 0, sizeof d);
    d.in_kind = RKB_IN_F16; d.out_kind = RKB_OUT_F16;
    d.M = M; d.N = N; d.K = K;
    d.A = A; d.lda = lda; d.B = W; d.ldb = K; d.C = C; d.ldc = ldc;
    d.bias = bias; d.act = act; d.residual = res; d.ldr = ldr;
    const size_t wb = rkb_gemm_workspace_bytes(&d);
    if (wb && !(d.workspace = enc_tmp(c, wb))) return;
    rkb_count(0, wb ? 2 : 1);
    int ps = rkb_prof_begin(c->h);
    enc_check(c, rkb_gemm_run(&d, c->h->err_dev, c->h->stream));
    rkb_prof_end(c->h, ps, RKB_K_GEMM_F16);
}

static int epi_act(int kind)
{
    if (kind == ROCKET_ACTIVATION_GELU) return RKB_ACT_GELU;
    if (kind == ROCKET_ACTIVATION_SILU) return RKB_ACT_SILU;
    return -1;
}

/* ---- norms / softmax --------------------------------------------------------- */
static int norm_common(const char *who, int fd, int M, int H, const void *x, const void *g,
                       const void *b, float eps, int rms, void *out)
{
    if (M < 1 || H < 1 || !x || !g || !out) return ROCKET_E_SHAPE;
    enc_call c;
    int rc = enc_begin(&c, fd, who);
    if (rc) return rc;
    const size_t bytes = (size_t)M * H * 2;
    const void *dx = enc_in(&c, x, bytes);
    const void *dg = enc_in(&c, g, (size_t)H * 2);
    const void *db = enc_in(&c, b, (size_t)H * 2);
    void *dout = enc_out(&c, out, bytes);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        enc_check(&c, rkb_norm_rows(dx, dg, db, M, H, eps, rms, dout, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_NORM);
        rkb_count(0, 1);
    }
    return enc_end(&c);
}

int rocket_layernorm_fp16(int fd, int M, int H, const _Float16 *x, const _Float16 *gamma,
                          const _Float16 *beta, float eps, _Float16 *out)
{
    return norm_common("rocket_layernorm_fp16", fd, M, H, x, gamma, beta, eps, 0, out);
}

int rocket_rmsnorm_fp16(int fd, int M, int H, const _Float16 *x, const _Float16 *weight, float eps,
                        _Float16 *out)
{
    return norm_common("rocket_rmsnorm_fp16", fd, M, H, x, weight, NULL, eps, 1, out);
}

static int softmax_common(const char *who, int fd, int M, int N, const void *in, void *out, int lg)
{
    if (M < 1 || N < 1 || !in || !out) return ROCKET_E_SHAPE;
    enc_call c;
    int rc = enc_begin(&c, fd, who);
    if (rc) return rc;
    const size_t bytes = (size_t)M * N * 2;
    const void *dx = enc_in(&c, in, bytes);
    void *dout = enc_out(&c, out, bytes);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        enc_check(&c, rkb_softmax_rows(dx, M, N, lg, dout, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_SOFTMAX);
        rkb_count(0, 1);
    }
    return enc_end(&c);
}

int rocket_softmax_fp16(int fd, int M, int N, const _Float16 *in, _Float16 *out)
{
    return softmax_common("rocket_softmax_fp16", fd, M, N, in, out, 0);
}

int rocket_logsoftmax_fp16(int fd, int M, int N, const _Float16 *in, _Float16 *out)
{
    return softmax_common("rocket_logsoftmax_fp16", fd, M, N, in, out, 1);
}

/* ---- element-wise ---------------------------------------------------------------- */
static int ew_common(const char *who, int fd, const void *a, const void *b, int op, int kind,
                     void *out, int n)
{
    if (n <= 0 || !a || !out || (op && !b)) return ROCKET_E_SHAPE;
    enc_call c;
    int rc = enc_begin(&c, fd, who);
    if (rc) return rc;
    const size_t bytes = (size_t)n * 2;
    const void *da = enc_in(&c, a, bytes);
    const void *db = op ? enc_in(&c, b, bytes) : NULL;
    void *dout = enc_out(&c, out, bytes);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        enc_check(&c, rkb_elementwise(da, db, op, kind, (size_t)n, dout, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_ELEMWISE);
        rkb_count(0, 1);
    }
    return enc_end(&c);
}

static int kind_ok(int kind)
{
    return kind >= 0 && kind <= 18 && kind != ROCKET_ACTIVATION_LEAKY_RELU &&
           kind != ROCKET_ACTIVATION_ELU && kind != ROCKET_ACTIVATION_SELU;
}

int rocket_activation_fp16(int fd, int kind, const _Float16 *in, _Float16 *out, int n)
{
    if (!kind_ok(kind)) {
        ROCKET_LOGE("rocket_activation_fp16: kind %d is parametric or unknown\n", kind);
        return ROCKET_E_UNSUPPORTED;
    }
    return ew_common("rocket_activation_fp16", fd, in, NULL, 0, kind, out, n);
}

int rocket_ew_add_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n)
{
    return ew_common("rocket_ew_add_fp16", fd, a, b, 1, 0, out, n);
}

int rocket_ew_mul_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n)
{
    return ew_common("rocket_ew_mul_fp16", fd, a, b, 2, 0, out, n);
}

int rocket_ew_sub_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n)
{
    return ew_common("rocket_ew_sub_fp16", fd, a, b, 3, 0, out, n);
}

int rocket_geglu_fp16(int fd, const _Float16 *gate, const _Float16 *up, int kind, _Float16 *prod, int n)
{
    if (!kind_ok(kind)) return ROCKET_E_UNSUPPORTED;
    return ew_common("rocket_geglu_fp16", fd, gate, up, 4, kind, prod, n);
}

/* ---- FFN / MLP ------------------------------------------------------------------------ */
int rocket_ffn_fp16(int fd, int M, int H, int I, const _Float16 *x, const _Float16 *Wg,
                    const _Float16 *Wu, const _Float16 *Wd, int kind, _Float16 *out)
{
    const char *who = "rocket_ffn_fp16";
    if (M < 1 || H < 1 || I < 1 || H % 32 || I % 32 || M % 4 || !x || !Wg || !Wu || !Wd || !out)
        return ROCKET_E_SHAPE;
    if (!kind_ok(kind)) return ROCKET_E_UNSUPPORTED;
    enc_call c;
    int rc = enc_begin(&c, fd, who);
    if (rc) return rc;
    const void *dx = enc_in(&c, x, (size_t)M * H * 2);
    const void *dwg = enc_in(&c, Wg, (size_t)I * H * 2);
    const void *dwu = enc_in(&c, Wu, (size_t)I * H * 2);
    const void *dwd = enc_in(&c, Wd, (size_t)H * I * 2);
    void *gate = enc_tmp(&c, (size_t)M * I * 2);
    void *up = enc_tmp(&c, (size_t)M * I * 2);
    void *dout = enc_out(&c, out, (size_t)M * H * 2);
    enc_gemm(&c, M, I, H, dx, H, dwg, gate, I, NULL, RKB_ACT_NONE, NULL, 0);
    enc_gemm(&c, M, I, H, dx, H, dwu, up, I, NULL, RKB_ACT_NONE, NULL, 0);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        enc_check(&c, rkb_elementwise(gate, up, 4, kind, (size_t)M * I, gate, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_ELEMWISE);
    }
    enc_gemm(&c, M, H, I, gate, I, dwd, dout, H, NULL, RKB_ACT_NONE, NULL, 0);
    return enc_end(&c);
}

int rocket_ffn_fp16_fused(int fd, int M, int H, int I, const _Float16 *x, const _Float16 *Wg,
                          const _Float16 *Wu, const _Float16 *Wd, int kind, _Float16 *out)
{
    return rocket_ffn_fp16(fd, M, H, I, x, Wg, Wu, Wd, kind, out);
}

int rocket_mlp_fp16_fused(int fd, int M, int Din, int Dff, int Dout, const _Float16 *x,
                          const _Float16 *W1, const _Float16 *b1, const _Float16 *W2, int kind,
                          _Float16 *out)
{
    const char *who = "rocket_mlp_fp16_fused";
    if (M < 1 || Din % 32 || Dff % 32 || Dout % 16 || M % 4 || Din < 1 || Dff < 1 || Dout < 1 ||
        !x || !W1 || !W2 || !out)
        return ROCKET_E_SHAPE;
    if (!kind_ok(kind)) return ROCKET_E_UNSUPPORTED;
    enc_call c;
    int rc = enc_begin(&c, fd, who);
    if (rc) return rc;
    const void *dx = enc_in(&c, x, (size_t)M * Din * 2);
    const void *dw1 = enc_in(&c, W1, (size_t)Dff * Din * 2);
    const void *db1 = enc_in(&c, b1, (size_t)Dff * 2);
    const void *dw2 = enc_in(&c, W2, (size_t)Dout * Dff * 2);
    void *f1 = enc_tmp(&c, (size_t)M * Dff * 2);
    void *dout = enc_out(&c, out, (size_t)M * Dout * 2);
    const int ea = epi_act(kind);
    enc_gemm(&c, M, Dff, Din, dx, Din, dw1, f1, Dff, db1, ea < 0 ? RKB_ACT_NONE : ea, NULL, 0);
    if (ea < 0 && !c.rc) enc_check(&c, rkb_elementwise(f1, NULL, 0, kind, (size_t)M * Dff, f1, c.h->stream));
    enc_gemm(&c, M, Dout, Dff, f1, Dff, dw2, dout, Dout, NULL, RKB_ACT_NONE, NULL, 0);
    return enc_end(&c);
}

/* ---- attention ------------------------------------------------------------------------- */
/* ctx[nb*T, d] = MHA core over nb sequences from ln[nb*T, d] (q/k/v projections included) */
static void enc_mha_core(enc_call *c, int nb, int T, int d, int n_head, const void *ln,
                         const void *Wq, const void *bq, const void *Wk, const void *bk,
                         const void *Wv, const void *bv, void *ctx)
{
    if (c->rc) return;
    const int BT = nb * T, dh = d / n_head, Tp = (T + 127) / 128 * 128;
    void *qkv = enc_tmp(c, (size_t)BT * 3 * d * 2);
    const size_t hsz = (size_t)nb * n_head * Tp * dh * 2;
    void *Q = enc_tmp(c, hsz), *K = enc_tmp(c, hsz), *Vt = enc_tmp(c, hsz);
    if (c->rc) return;
    enc_gemm(c, BT, d, d, ln, d, Wq, qkv, 3 * d, bq, RKB_ACT_NONE, NULL, 0);
    enc_gemm(c, BT, d, d, ln, d, Wk, (uint8_t *)qkv + (size_t)d * 2, 3 * d, bk, RKB_ACT_NONE, NULL, 0);
    enc_gemm(c, BT, d, d, ln, d, Wv, (uint8_t *)qkv + (size_t)2 * d * 2, 3 * d, bv, RKB_ACT_NONE, NULL, 0);
    if (c->rc) return;
    int ps = rkb_prof_begin(c->h);
    enc_check(c, rkb_split_heads(qkv, 3 * d, nb, T, Tp, n_head, dh, Q, K, Vt, c->h->stream));
    rkb_prof_end(c->h, ps, RKB_K_ELEMWISE);
    ps = rkb_prof_begin(c->h);
    if (!c->rc)
        enc_check(c, rkb_attention(Q, K, Vt, nb, n_head, T, Tp, dh, 1.0f / sqrtf((float)dh), ctx, d,
                                   c->h->err_dev, c->h->stream));
    rkb_prof_end(c->h, ps, RKB_K_ATTN);
    rkb_count(0, 2);
}

static int mha_shape_ok(int T, int d, int n_head)
{
    return T >= 1 && d >= 1 && n_head >= 1 && d % n_head == 0 && d % 32 == 0;
}

int rocket_mha_self_fp16(int fd, int T, int d, int n_head, const _Float16 *x, const _Float16 *Wq,
                         const _Float16 *bq, const _Float16 *Wk, const _Float16 *bk,
                         const _Float16 *Wv, const _Float16 *bv, const _Float16 *Wo,
                         const _Float16 *bo, _Float16 *out)
{
    const char *who = "rocket_mha_self_fp16";
    if (!mha_shape_ok(T, d, n_head) || !x || !Wq || !Wk || !Wv || !Wo || !out) return ROCKET_E_SHAPE;
    if (d / n_head != 64) {
        ROCKET_LOGE("%s: head_dim %d unsupported (the fused kernel is built for 64)\n", who, d / n_head);
        return ROCKET_E_UNSUPPORTED;
    }
    enc_call c;
    int rc = enc_begin(&c, fd, who);
    if (rc) return rc;
    const size_t w = (size_t)d * d * 2, v = (size_t)d * 2, a = (size_t)T * d * 2;
    const void *dx = enc_in(&c, x, a);
    const void *dq = enc_in(&c, Wq, w), *dk = enc_in(&c, Wk, w), *dv = enc_in(&c, Wv, w), *dwo = enc_in(&c, Wo, w);
    const void *dbq = enc_in(&c, bq, v), *dbk = enc_in(&c, bk, v), *dbv = enc_in(&c, bv, v), *dbo = enc_in(&c, bo, v);
    void *ctx = enc_tmp(&c, a);
    void *dout = enc_out(&c, out, a);
    enc_mha_core(&c, 1, T, d, n_head, dx, dq, dbq, dk, dbk, dv, dbv, ctx);
    enc_gemm(&c, T, d, d, ctx, d, dwo, dout, d, dbo, RKB_ACT_NONE, NULL, 0);
    return enc_end(&c);
}

/* ---- encoder block ------------------------------------------------------------------- */
static int encoder_common(const char *who, int fd, int nb, int T, int d, int n_head, int d_ff,
                          const void *x, const void *ln1_g, const void *ln1_b, const void *Wq,
                          const void *bq, const void *Wk, const void *bk, const void *Wv,
                          const void *bv, const void *Wo, const void *bo, const void *ln2_g,
                          const void *ln2_b, const void *Wf1, const void *bf1, const void *Wf2,
                          const void *bf2, float eps, void *out)
{
    if (nb < 1 || !mha_shape_ok(T, d, n_head) || d_ff < 1 || d_ff % 8 || !x || !ln1_g || !ln2_g ||
        !Wq || !Wk || !Wv || !Wo || !Wf1 || !Wf2 || !out)
        return ROCKET_E_SHAPE;
    if (d / n_head != 64) {
        ROCKET_LOGE("%s: head_dim %d unsupported (the fused kernel is built for 64)\n", who, d / n_head);
        return ROCKET_E_UNSUPPORTED;
    }
    enc_call c;
    int rc = enc_begin(&c, fd, who);
    if (rc) return rc;
    const int BT = nb * T;
    const size_t act = (size_t)BT * d * 2, w = (size_t)d * d * 2, v = (size_t)d * 2;
    const void *dx = enc_in(&c, x, act);
    const void *g1 = enc_in(&c, ln1_g, v), *b1 = enc_in(&c, ln1_b, v);
    const void *g2 = enc_in(&c, ln2_g, v), *b2 = enc_in(&c, ln2_b, v);
    const void *dq = enc_in(&c, Wq, w), *dk = enc_in(&c, Wk, w), *dv = enc_in(&c, Wv, w), *dwo = enc_in(&c, Wo, w);
    const void *dbq = enc_in(&c, bq, v), *dbk = enc_in(&c, bk, v), *dbv = enc_in(&c, bv, v), *dbo = enc_in(&c, bo, v);
    const void *dw1 = enc_in(&c, Wf1, (size_t)d_ff * d * 2), *dbf1 = enc_in(&c, bf1, (size_t)d_ff * 2);
    const void *dw2 = enc_in(&c, Wf2, (size_t)d * d_ff * 2), *dbf2 = enc_in(&c, bf2, v);
    void *ln = enc_tmp(&c, act), *ctx = enc_tmp(&c, act), *xa = enc_tmp(&c, act);
    void *f1 = enc_tmp(&c, (size_t)BT * d_ff * 2);
    void *dout = enc_out(&c, out, act);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        enc_check(&c, rkb_norm_rows(dx, g1, b1, BT, d, eps, 0, ln, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_NORM);
    }
    enc_mha_core(&c, nb, T, d, n_head, ln, dq, dbq, dk, dbk, dv, dbv, ctx);
    enc_gemm(&c, BT, d, d, ctx, d, dwo, xa, d, dbo, RKB_ACT_NONE, dx, d);          /* x + MHA */
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        enc_check(&c, rkb_norm_rows(xa, g2, b2, BT, d, eps, 0, ln, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_NORM);
    }
    enc_gemm(&c, BT, d_ff, d, ln, d, dw1, f1, d_ff, dbf1, RKB_ACT_GELU, NULL, 0);  /* GELU(fc1) */
    enc_gemm(&c, BT, d, d_ff, f1, d_ff, dw2, dout, d, dbf2, RKB_ACT_NONE, xa, d);  /* + residual */
    rkb_count(0, 2);
    return enc_end(&c);
}

int rocket_encoder_block_fp16(int fd, int T, int d, int n_head, int d_ff, const _Float16 *x,
                              const _Float16 *ln1_g, const _Float16 *ln1_b, const _Float16 *Wq,
                              const _Float16 *bq, const _Float16 *Wk, const _Float16 *bk,
                              const _Float16 *Wv, const _Float16 *bv, const _Float16 *Wo,
                              const _Float16 *bo, const _Float16 *ln2_g, const _Float16 *ln2_b,
                              const _Float16 *Wf1, const _Float16 *bf1, const _Float16 *Wf2,
                              const _Float16 *bf2, float eps, _Float16 *out)
{
    return encoder_common("rocket_encoder_block_fp16", fd, 1, T, d, n_head, d_ff, x, ln1_g, ln1_b,
                          Wq, bq, Wk, bk, Wv, bv, Wo, bo, ln2_g, ln2_b, Wf1, bf1, Wf2, bf2, eps, out);
}

int rocket_b200_encoder_block_batched_fp16(int fd, int nb, int T, int d, int n_head, int d_ff,
                                           const void *x, const void *ln1_g, const void *ln1_b,
                                           const void *Wq, const void *bq, const void *Wk,
                                           const void *bk, const void *Wv, const void *bv,
                                           const void *Wo, const void *bo, const void *ln2_g,
                                           const void *ln2_b, const void *Wf1, const void *bf1,
                                           const void *Wf2, const void *bf2, float eps, void *out)
{
    return encoder_common("rocket_b200_encoder_block_batched_fp16", fd, nb, T, d, n_head, d_ff, x,
                          ln1_g, ln1_b, Wq, bq, Wk, bk, Wv, bv, Wo, bo, ln2_g, ln2_b, Wf1, bf1, Wf2,
                          bf2, eps, out);
}
