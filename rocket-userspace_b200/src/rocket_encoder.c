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
#include "rocket_reduce.h"
#include "rocket_softmax.h"
#include "rkb_internal.h"

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
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const size_t bytes = (size_t)M * H * 2;
    const void *dx = rkb_call_in(&c, x, bytes);
    const void *dg = rkb_call_in(&c, g, (size_t)H * 2);
    const void *db = rkb_call_in(&c, b, (size_t)H * 2);
    void *dout = rkb_call_out(&c, out, bytes);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        rkb_call_check(&c, rkb_norm_rows(dx, dg, db, M, H, eps, rms, dout, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_NORM);
        rkb_count(0, 1);
    }
    return rkb_call_end(&c);
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
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const size_t bytes = (size_t)M * N * 2;
    const void *dx = rkb_call_in(&c, in, bytes);
    void *dout = rkb_call_out(&c, out, bytes);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        rkb_call_check(&c, rkb_softmax_rows(dx, M, N, lg, dout, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_SOFTMAX);
        rkb_count(0, 1);
    }
    return rkb_call_end(&c);
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
static int ew_common2(const char *who, int fd, const void *a, const void *b, int op, int kind,
                      float lo, float hi, void *out, int n)
{
    const int two = op >= 1 && op <= 6;
    if (n <= 0 || !a || !out || (two && !b)) return ROCKET_E_SHAPE;
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const size_t bytes = (size_t)n * 2;
    const void *da = rkb_call_in(&c, a, bytes);
    const void *db = two ? rkb_call_in(&c, b, bytes) : NULL;
    void *dout = rkb_call_out(&c, out, bytes);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        rkb_call_check(&c, rkb_elementwise_ex(da, db, op, kind, lo, hi, (size_t)n, dout, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_ELEMWISE);
        rkb_count(0, 1);
    }
    return rkb_call_end(&c);
}

static int ew_common(const char *who, int fd, const void *a, const void *b, int op, int kind,
                     void *out, int n)
{
    return ew_common2(who, fd, a, b, op, kind, 0.f, 0.f, out, n);
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

/* max / min / clip (reference include/rocket_activation.h:170-178): one
 * element-wise kernel each; clip is a single pass min(max(x, lo), hi). */
int rocket_ew_max_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n)
{
    return ew_common("rocket_ew_max_fp16", fd, a, b, 5, 0, out, n);
}

int rocket_ew_min_fp16(int fd, const _Float16 *a, const _Float16 *b, _Float16 *out, int n)
{
    return ew_common("rocket_ew_min_fp16", fd, a, b, 6, 0, out, n);
}

int rocket_clip_fp16(int fd, float lo, float hi, const _Float16 *in, _Float16 *out, int n)
{
    if (!(lo <= hi)) return ROCKET_E_SHAPE;
    return ew_common2("rocket_clip_fp16", fd, in, NULL, 7, 0, lo, hi, out, n);
}

/* Names as the reference prints them (src/rocket_activation.c:116-140). */
const char *rocket_activation_name(int kind)
{
    static const char *const names[] = {
        "sigmoid", "hardsigmoid", "hardswish", "silu", "tanh", "gelu", "leaky_relu", "sqrt",
        "rsqrt", "reciprocal", "exp", "gelu_gate", "softplus", "mish_gate", "mish", "abs",
        "elu", "selu", "log"};
    return kind >= 0 && kind < (int)(sizeof names / sizeof names[0]) ? names[kind] : "?";
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
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const void *dx = rkb_call_in(&c, x, (size_t)M * H * 2);
    const void *dwg = rkb_call_in(&c, Wg, (size_t)I * H * 2);
    const void *dwu = rkb_call_in(&c, Wu, (size_t)I * H * 2);
    const void *dwd = rkb_call_in(&c, Wd, (size_t)H * I * 2);
    void *gate = rkb_call_tmp(&c, (size_t)M * I * 2);
    void *up = rkb_call_tmp(&c, (size_t)M * I * 2);
    void *dout = rkb_call_out(&c, out, (size_t)M * H * 2);
    rkb_call_gemm(&c, M, I, H, dx, H, dwg, gate, I, NULL, RKB_ACT_NONE, NULL, 0);
    rkb_call_gemm(&c, M, I, H, dx, H, dwu, up, I, NULL, RKB_ACT_NONE, NULL, 0);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        rkb_call_check(&c, rkb_elementwise(gate, up, 4, kind, (size_t)M * I, gate, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_ELEMWISE);
    }
    rkb_call_gemm(&c, M, H, I, gate, I, dwd, dout, H, NULL, RKB_ACT_NONE, NULL, 0);
    return rkb_call_end(&c);
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
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const void *dx = rkb_call_in(&c, x, (size_t)M * Din * 2);
    const void *dw1 = rkb_call_in(&c, W1, (size_t)Dff * Din * 2);
    const void *db1 = rkb_call_in(&c, b1, (size_t)Dff * 2);
    const void *dw2 = rkb_call_in(&c, W2, (size_t)Dout * Dff * 2);
    void *f1 = rkb_call_tmp(&c, (size_t)M * Dff * 2);
    void *dout = rkb_call_out(&c, out, (size_t)M * Dout * 2);
    const int ea = epi_act(kind);
    rkb_call_gemm(&c, M, Dff, Din, dx, Din, dw1, f1, Dff, db1, ea < 0 ? RKB_ACT_NONE : ea, NULL, 0);
    if (ea < 0 && !c.rc) rkb_call_check(&c, rkb_elementwise(f1, NULL, 0, kind, (size_t)M * Dff, f1, c.h->stream));
    rkb_call_gemm(&c, M, Dout, Dff, f1, Dff, dw2, dout, Dout, NULL, RKB_ACT_NONE, NULL, 0);
    return rkb_call_end(&c);
}

/* ---- attention ------------------------------------------------------------------------- */
/* The q / k / v projections run as one GEMM of N = 3d: the three weights are
 * staged into one [3d, d] buffer (and the biases into one [3d] vector; a NULL
 * bias is zeros, all three NULL is no bias), which fills the GPU's SM pairs
 * better than three N = d GEMMs and saves two launches. */
static void enc_stage_qkv(rkb_call *c, int d, const void *Wq, const void *Wk, const void *Wv,
                          const void *bq, const void *bk, const void *bv, void **wqkv, void **bqkv)
{
    *wqkv = NULL;
    *bqkv = NULL;
    if (c->rc) return;
    const size_t w = (size_t)d * d * 2, v = (size_t)d * 2;
    uint8_t *dw = rkb_call_tmp(c, 3 * w);
    uint8_t *db = (bq || bk || bv) ? rkb_call_tmp(c, 3 * v) : NULL;
    if (c->rc) return;
    const void *ws[3] = {Wq, Wk, Wv}, *bs[3] = {bq, bk, bv};
    /* device-resident, aligned inputs: one gather kernel for the weights, one for the biases */
    int on_dev = 1;
    for (int i = 0; i < 3; i++) {
        if (rkb_ptr_device(ws[i]) != c->h->device || ((uintptr_t)ws[i] & 15)) on_dev = 0;
        if (bs[i] && (rkb_ptr_device(bs[i]) != c->h->device || ((uintptr_t)bs[i] & 15))) on_dev = 0;
    }
    if (on_dev && v % 16 == 0) {
        rkb_call_check(c, rkb_concat3(Wq, Wk, Wv, w, dw, c->h->stream));
        if (db) rkb_call_check(c, rkb_concat3(bq, bk, bv, v, db, c->h->stream));
        rkb_count(0, db ? 2 : 1);
        *wqkv = dw;
        *bqkv = db;
        return;
    }
    for (int i = 0; i < 3; i++)
        if (rkb_ptr_device(ws[i]) < 0 || (bs[i] && rkb_ptr_device(bs[i]) < 0)) c->host_in = 1;
    for (int i = 0; i < 3 && !c->rc; i++) {
        if (cudaMemcpyAsync(dw + i * w, ws[i], w, cudaMemcpyDefault, c->h->stream) != cudaSuccess) {
            cudaGetLastError();
            c->rc = ROCKET_E_DEVICE;
        }
        if (db && !c->rc) {
            cudaError_t e = bs[i] ? cudaMemcpyAsync(db + i * v, bs[i], v, cudaMemcpyDefault, c->h->stream)
                                  : cudaMemsetAsync(db + i * v, 0, v, c->h->stream);
            if (e != cudaSuccess) {
                cudaGetLastError();
                c->rc = ROCKET_E_DEVICE;
            }
        }
    }
    *wqkv = dw;
    *bqkv = db;
}

/* ctx[nb*T, d] = MHA core over nb sequences from ln[nb*T, d] (q/k/v projection included) */
static void enc_mha_core(rkb_call *c, int nb, int T, int d, int n_head, const void *ln,
                         const void *Wqkv, const void *bqkv, void *ctx)
{
    if (c->rc) return;
    const int BT = nb * T, dh = d / n_head, Tp = (T + 127) / 128 * 128;
    void *qkv = rkb_call_tmp(c, (size_t)BT * 3 * d * 2);
    const size_t hsz = (size_t)nb * n_head * Tp * dh * 2;
    void *Q = rkb_call_tmp(c, hsz), *K = rkb_call_tmp(c, hsz), *Vt = rkb_call_tmp(c, hsz);
    if (c->rc) return;
    rkb_call_gemm(c, BT, 3 * d, d, ln, d, Wqkv, qkv, 3 * d, bqkv, RKB_ACT_NONE, NULL, 0);
    if (c->rc) return;
    int ps = rkb_prof_begin(c->h);
    rkb_call_check(c, rkb_split_heads(qkv, 3 * d, nb, T, Tp, n_head, dh, Q, K, Vt, c->h->stream));
    rkb_prof_end(c->h, ps, RKB_K_ELEMWISE);
    ps = rkb_prof_begin(c->h);
    /* head_dim 64: the register-resident-O kernel; other head dims: the flash
     * kernel over the same split heads (nb * n_head heads of Tp rows, output
     * interleaved back into ctx[token][head * dh]) */
    static int force_fa = -1;
    if (force_fa < 0) force_fa = (int)rkb_env_long("ROCKET_ATTN_FA", 0);
    if (!c->rc && dh == 64 && !force_fa)
        rkb_call_check(c, rkb_attention(Q, K, Vt, nb, n_head, T, Tp, dh, 1.0f / sqrtf((float)dh), ctx, d,
                                   c->h->err_dev, c->h->stream));
    else if (!c->rc)
        rkb_call_check(c, rkb_flash_attn_ex(Q, K, Vt, Tp, NULL, ctx, T, T, dh, dh, nb * n_head, nb * n_head,
                                            1.0f / sqrtf((float)dh), 0.0f, Tp, Tp, n_head, (long)T * d, d,
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
    if ((d / n_head) % 16 || d / n_head > 256) {
        ROCKET_LOGE("%s: head_dim %d unsupported (needs a multiple of 16, at most 256)\n", who, d / n_head);
        return ROCKET_E_UNSUPPORTED;
    }
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const size_t w = (size_t)d * d * 2, v = (size_t)d * 2, a = (size_t)T * d * 2;
    const void *dx = rkb_call_in(&c, x, a);
    const void *dwo = rkb_call_in(&c, Wo, w), *dbo = rkb_call_in(&c, bo, v);
    void *wqkv, *bqkv;
    enc_stage_qkv(&c, d, Wq, Wk, Wv, bq, bk, bv, &wqkv, &bqkv);
    void *ctx = rkb_call_tmp(&c, a);
    void *dout = rkb_call_out(&c, out, a);
    enc_mha_core(&c, 1, T, d, n_head, dx, wqkv, bqkv, ctx);
    rkb_call_gemm(&c, T, d, d, ctx, d, dwo, dout, d, dbo, RKB_ACT_NONE, NULL, 0);
    return rkb_call_end(&c);
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
    if ((d / n_head) % 16 || d / n_head > 256) {
        ROCKET_LOGE("%s: head_dim %d unsupported (needs a multiple of 16, at most 256)\n", who, d / n_head);
        return ROCKET_E_UNSUPPORTED;
    }
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const int BT = nb * T;
    const size_t act = (size_t)BT * d * 2, w = (size_t)d * d * 2, v = (size_t)d * 2;
    const void *dx = rkb_call_in(&c, x, act);
    const void *g1 = rkb_call_in(&c, ln1_g, v), *b1 = rkb_call_in(&c, ln1_b, v);
    const void *g2 = rkb_call_in(&c, ln2_g, v), *b2 = rkb_call_in(&c, ln2_b, v);
    const void *dwo = rkb_call_in(&c, Wo, w), *dbo = rkb_call_in(&c, bo, v);
    void *wqkv, *bqkv;
    enc_stage_qkv(&c, d, Wq, Wk, Wv, bq, bk, bv, &wqkv, &bqkv);
    const void *dw1 = rkb_call_in(&c, Wf1, (size_t)d_ff * d * 2), *dbf1 = rkb_call_in(&c, bf1, (size_t)d_ff * 2);
    const void *dw2 = rkb_call_in(&c, Wf2, (size_t)d * d_ff * 2), *dbf2 = rkb_call_in(&c, bf2, v);
    void *ln = rkb_call_tmp(&c, act), *ctx = rkb_call_tmp(&c, act), *xa = rkb_call_tmp(&c, act);
    void *f1 = rkb_call_tmp(&c, (size_t)BT * d_ff * 2);
    void *dout = rkb_call_out(&c, out, act);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        rkb_call_check(&c, rkb_norm_rows(dx, g1, b1, BT, d, eps, 0, ln, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_NORM);
    }
    enc_mha_core(&c, nb, T, d, n_head, ln, wqkv, bqkv, ctx);
    rkb_call_gemm(&c, BT, d, d, ctx, d, dwo, xa, d, dbo, RKB_ACT_NONE, dx, d);          /* x + MHA */
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        rkb_call_check(&c, rkb_norm_rows(xa, g2, b2, BT, d, eps, 0, ln, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_NORM);
    }
    rkb_call_gemm(&c, BT, d_ff, d, ln, d, dw1, f1, d_ff, dbf1, RKB_ACT_GELU, NULL, 0);  /* GELU(fc1) */
    rkb_call_gemm(&c, BT, d, d_ff, f1, d_ff, dw2, dout, d, dbf2, RKB_ACT_NONE, xa, d);  /* + residual */
    rkb_count(0, 2);
    return rkb_call_end(&c);
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

/* ---- reductions ---------------------------------------------------------------------------
 * Reference: src/rocket_reduce.c:380-510 (feature reduce, cumsum via ones / triangular
 * matmuls), src/rocket_norm.c:21-60 (scale_rows), src/rocket_softmax.c:141-190 (cross
 * entropy).  Each is one warp-per-row (or element-wise) pass in fp32. */
int rocket_reduce_feature_fp16(int fd, int M, int H, const _Float16 *in, float *out, int mean)
{
    if (M < 1 || H < 1 || !in || !out) return ROCKET_E_SHAPE;
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, "rocket_reduce_feature_fp16");
    if (rc) return rc;
    const void *dx = rkb_call_in(&c, in, (size_t)M * H * 2);
    float *dout = rkb_call_out(&c, out, (size_t)M * 4);
    if (!c.rc) rkb_call_check(&c, rkb_reduce_rows(dx, M, H, mean, dout, c.h->stream));
    return rkb_call_end(&c);
}

int rocket_cumsum_fp16(int fd, int M, int N, const _Float16 *in, _Float16 *out, int exclusive, int reverse)
{
    if (M < 1 || N < 1 || !in || !out) return ROCKET_E_SHAPE;
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, "rocket_cumsum_fp16");
    if (rc) return rc;
    const void *dx = rkb_call_in(&c, in, (size_t)M * N * 2);
    void *dout = rkb_call_out(&c, out, (size_t)M * N * 2);
    if (!c.rc) rkb_call_check(&c, rkb_cumsum_rows(dx, M, N, exclusive, reverse, dout, c.h->stream));
    return rkb_call_end(&c);
}

int rocket_scale_rows_fp16(int fd, int M, int N, const _Float16 *in, const float *r, _Float16 *out)
{
    if (M < 1 || N < 1 || !in || !r || !out) return ROCKET_E_SHAPE;
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, "rocket_scale_rows_fp16");
    if (rc) return rc;
    const void *dx = rkb_call_in(&c, in, (size_t)M * N * 2);
    const float *dr = rkb_call_in(&c, r, (size_t)M * 4);
    void *dout = rkb_call_out(&c, out, (size_t)M * N * 2);
    if (!c.rc) rkb_call_check(&c, rkb_scale_rows(dx, dr, M, N, dout, c.h->stream));
    return rkb_call_end(&c);
}

int rocket_cross_entropy_fp16(int fd, int M, int N, const _Float16 *logits, const int *target, float *loss)
{
    if (M < 1 || N < 1 || !logits || !target || !loss) return ROCKET_E_SHAPE;
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, "rocket_cross_entropy_fp16");
    if (rc) return rc;
    const void *dx = rkb_call_in(&c, logits, (size_t)M * N * 2);
    const int *dt = rkb_call_in(&c, target, (size_t)M * 4);
    float *dl = rkb_call_out(&c, loss, (size_t)M * 4);
    if (!c.rc) rkb_call_check(&c, rkb_cross_entropy_rows(dx, dt, M, N, dl, c.h->stream));
    return rkb_call_end(&c);
}
