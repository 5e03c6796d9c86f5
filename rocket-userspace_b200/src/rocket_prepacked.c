/*
 * rocket_prepacked.c -- resident weights and the multi-GPU N-split.
 *
 * Reference: src/rocket_prepacked.c:79-447 (fp16 ctx / weights),
 * src/rocket_prepacked_int8.c:140-767 (W8A8, per-channel and group-wise),
 * src/rocket_prepacked_int4.c:98-686 (W4A4) and src/rocket_matmul_mt.c:58-99.
 *
 * The reference's worker = one NPU fd driven by one pthread, computing
 * C[:, n0:n0+nsub] from the full A.  Here a worker = one device handle (one GPU
 * and its stream); worker t runs on GPU t % ndev.  The slice split is the
 * reference's (ceil(N / nthreads) rounded up to the dtype's N atom: 16 fp16,
 * 32 int8, 64 int4).  One host thread drives every worker asynchronously --
 * stage A into each GPU, launch, copy each slice into C -- and then waits for
 * all of them, so no pthread per call is needed: a GPU launch does not block
 * the host the way an NPU fence wait does.
 *
 * Weights live on their worker's GPU in the layout the kernel reads directly:
 *   fp16 / int8 per-channel   row-major slice [nsub, K] (TMA tiles it)
 *   int8 / int4 group-wise    tiled offset-binary codes (rkb_wpack_codes)
 *   int4 per-channel          tiled nibble codes, widened to int8 in registers
 * Because none of these depends on M, the reference's "-2: re-pack for this M"
 * case never arises; K or N differing from the pack returns ROCKET_E_SHAPE.
 */
#include <stdlib.h>
#include <string.h>

#include "rocket_matmul.h"
#include "rocket_b200.h"
#include "rkb_internal.h"

typedef enum { RW_F16, RW_I8, RW_I8_GW, RW_I4, RW_I4_GW, RW_BF16 } rw_kind;

typedef struct {
    int nthreads;
    int atom;                       /* N alignment of a slice */
    int fd[RKB_MAX_WORKERS];
} rkb_rctx;

typedef struct {
    rw_kind kind;
    int M, K, N, group, nt;
    int n0[RKB_MAX_WORKERS], nsub[RKB_MAX_WORKERS];
    void *dev[RKB_MAX_WORKERS];
    size_t bytes[RKB_MAX_WORKERS];
    size_t cap[RKB_MAX_WORKERS];
} rkb_rweights;

struct rocket_ctx        { rkb_rctx r; };
struct rocket_weights    { rkb_rweights w; };
struct rocket_i8_ctx     { rkb_rctx r; };
struct rocket_i8_weights { rkb_rweights w; };
struct rocket_i4_ctx     { rkb_rctx r; };
struct rocket_i4_weights { rkb_rweights w; };

/* ---- ctx ------------------------------------------------------------------ */
static int rctx_init(rkb_rctx *c, int nthreads, int atom, const char *who)
{
    if (nthreads < 1) nthreads = 1;
    if (nthreads > RKB_MAX_WORKERS) nthreads = RKB_MAX_WORKERS;
    int ndev = rkb_device_count();
    if (ndev <= 0) {
        ROCKET_LOGE("%s: no CUDA device\n", who);
        return ROCKET_E_DEVICE;
    }
    c->nthreads = nthreads;
    c->atom = atom;
    const int base = (int)rkb_env_long("ROCKET_DEV", 0);
    for (int t = 0; t < nthreads; t++) {
        c->fd[t] = rkb_open_on((base + t) % ndev);
        if (c->fd[t] < 0) {
            ROCKET_LOGE("%s: open worker %d failed (%d)\n", who, t, c->fd[t]);
            for (int u = 0; u < t; u++) rocket_close(c->fd[u]);
            return ROCKET_E_DEVICE;
        }
    }
    /* let slices copy straight into a peer GPU's output buffer: peer access
     * between every pair of the devices the workers actually run on
     * ((base + t) % ndev), leaving the caller's current device as it was */
    int cur = 0;
    cudaGetDevice(&cur);
    const int nd = nthreads < ndev ? nthreads : ndev;
    for (int i = 0; i < nd; i++)
        for (int j = 0; j < nd; j++) {
            const int a = (base + i) % ndev, b = (base + j) % ndev;
            if (a == b) continue;
            int can = 0;
            cudaDeviceCanAccessPeer(&can, a, b);
            if (can) {
                cudaSetDevice(a);
                cudaDeviceEnablePeerAccess(b, 0);
                cudaGetLastError();   /* already enabled is fine */
            }
        }
    cudaSetDevice(cur);
    return 0;
}

int rocket_b200_ctx_fd(const void *ctx, int worker)
{
    const rkb_rctx *c = ctx;
    if (!c || worker < 0 || worker >= c->nthreads) return ROCKET_E_SHAPE;
    return c->fd[worker];
}

static void rctx_free_on(rkb_rctx *c)
{
    for (int t = 0; t < c->nthreads; t++) rocket_close(c->fd[t]);
}

/* reference slice rule (src/rocket_prepacked_int8.c:161-165) */
static int nstep(int N, int nthreads, int atom)
{
    int s = ((N + nthreads - 1) / nthreads + atom - 1) / atom * atom;
    return s < atom ? atom : s;
}

/* ---- weights ---------------------------------------------------------------- */
/* Fill w with the workers' N-slices of the weight.  The weight is given as nseg
 * row blocks Bs[i] of Ns[i] rows each (one block for a plain weight; several
 * for a fused N-concatenation).  Existing per-worker buffers large enough are
 * reused (the streaming contexts re-fill every call); finish = 0 leaves the
 * copies queued for the call that follows. */
static int rweights_fill_on(const rkb_rctx *c, rkb_rweights *w, rw_kind kind, int M, int K, int N, int nseg,
                         const void *const *Bs, const int *Ns, int group, int finish, const char *who)
{
    void *keep[RKB_MAX_WORKERS];
    size_t keep_cap[RKB_MAX_WORKERS];
    memcpy(keep, w->dev, sizeof keep);
    memcpy(keep_cap, w->cap, sizeof keep_cap);
    memset(w, 0, sizeof *w);
    memcpy(w->dev, keep, sizeof keep);
    memcpy(w->cap, keep_cap, sizeof keep_cap);
    w->kind = kind; w->M = M; w->K = K; w->N = N; w->group = group;
    const int step = nstep(N, c->nthreads, c->atom);
    const size_t esz = kind == RW_F16 ? 2 : kind == RW_BF16 ? 4 : 1;   /* caller's element size */
    const int gw = (kind == RW_I8_GW || kind == RW_I4_GW || kind == RW_I4);
    if (gw && nseg != 1) return ROCKET_E_SHAPE;
    int rc = 0;
    for (int t = 0; t < c->nthreads && !rc; t++) {
        const int n0 = t * step;
        const int nsub = n0 >= N ? 0 : (N - n0 < step ? N - n0 : step);
        w->n0[t] = n0;
        w->nsub[t] = nsub;
        if (nsub <= 0) continue;
        w->nt = t + 1;
        rkb_handle *h = rkb_get(c->fd[t]);
        const size_t raw = (size_t)nsub * K * esz;
        size_t need;
        if (gw) need = rkb_wpack_codes_bytes(nsub, K, kind == RW_I8_GW ? 8 : 4);
        else if (kind == RW_BF16) need = (size_t)nsub * K * 2;
        else need = raw;
        w->bytes[t] = need;
        if (w->cap[t] < need) {
            if (w->dev[t]) { cudaStreamSynchronize(h->stream); cudaFree(w->dev[t]); }
            w->dev[t] = NULL;
            w->cap[t] = 0;
            if (cudaMalloc(&w->dev[t], need) != cudaSuccess) { cudaGetLastError(); rc = ROCKET_E_NOMEM; break; }
            w->cap[t] = need;
        }
        if (gw) {
            const void *src = (const uint8_t *)Bs[0] + (size_t)n0 * K;
            const void *dsrc = rkb_stage_in(h, RKB_SCR_B, src, raw);
            if (!dsrc) { rc = ROCKET_E_NOMEM; break; }
            int ps = rkb_prof_begin(h);
            rc = rkb_wpack_codes(dsrc, nsub, K, kind == RW_I8_GW ? 8 : 4, w->dev[t], h->stream);
            rkb_prof_end(h, ps, RKB_K_PACK);
        } else {
            /* gather the slice rows [n0, n0+nsub) from the segments */
            uint8_t *dst = w->dev[t];
            if (kind == RW_BF16) dst = rkb_scratch(h, RKB_SCR_B, raw);   /* fp32 staging */
            if (!dst) { rc = ROCKET_E_NOMEM; break; }
            int base = 0;
            for (int sg = 0; sg < nseg && !rc; sg++) {
                const int lo = n0 > base ? n0 : base;
                const int hi = (n0 + nsub) < (base + Ns[sg]) ? (n0 + nsub) : (base + Ns[sg]);
                if (hi > lo) {
                    const uint8_t *src = (const uint8_t *)Bs[sg] + (size_t)(lo - base) * K * esz;
                    if (cudaMemcpyAsync(dst + (size_t)(lo - n0) * K * esz, src, (size_t)(hi - lo) * K * esz,
                                        cudaMemcpyDefault, h->stream) != cudaSuccess) {
                        cudaGetLastError();
                        rc = ROCKET_E_DEVICE;
                    }
                }
                base += Ns[sg];
            }
            if (!rc && kind == RW_BF16) rc = rkb_f32_to_bf16(dst, (size_t)nsub * K, w->dev[t], h->stream);
        }
        rkb_count(1, 1);
    }
    if (finish || rc) {
        for (int t = 0; t < w->nt; t++) {
            int fr = rkb_finish(rkb_get(c->fd[t]), who);
            if (!rc) rc = fr;
        }
    }
    if (rc) ROCKET_LOGE("%s: weight upload failed (%d)\n", who, rc);
    return rc;
}

static void rweights_free_on(const rkb_rctx *c, rkb_rweights *w);

/* The workers switch the current CUDA device; every entry point leaves the
 * caller's current device as it found it. */
static int rweights_fill(const rkb_rctx *c, rkb_rweights *w, rw_kind kind, int M, int K, int N, int nseg,
                         const void *const *Bs, const int *Ns, int group, int finish, const char *who)
{
    int dev0 = 0;
    cudaGetDevice(&dev0);
    int rc = rweights_fill_on(c, w, kind, M, K, N, nseg, Bs, Ns, group, finish, who);
    cudaSetDevice(dev0);
    return rc;
}

static void rweights_free(const rkb_rctx *c, rkb_rweights *w)
{
    int dev0 = 0;
    cudaGetDevice(&dev0);
    rweights_free_on(c, w);
    cudaSetDevice(dev0);
}

static void rctx_free(rkb_rctx *c)
{
    int dev0 = 0;
    cudaGetDevice(&dev0);
    rctx_free_on(c);
    cudaSetDevice(dev0);
}

static int rweights_pack(const rkb_rctx *c, rkb_rweights *w, rw_kind kind, int M, int K, int N,
                         const void *B, int group, const char *who)
{
    memset(w, 0, sizeof *w);
    const void *bs[1] = {B};
    const int ns[1] = {N};
    int rc = rweights_fill(c, w, kind, M, K, N, 1, bs, ns, group, 1, who);
    if (rc) rweights_free(c, w);
    return rc;
}

static void rweights_free_on(const rkb_rctx *c, rkb_rweights *w)
{
    for (int t = 0; t < c->nthreads; t++) {
        if (!w->dev[t]) continue;
        rkb_handle *h = rkb_get(c->fd[t]);
        if (h) cudaStreamSynchronize(h->stream);
        cudaFree(w->dev[t]);
        w->dev[t] = NULL;
        w->cap[t] = 0;
    }
}

static size_t rweights_bytes(const rkb_rweights *w)
{
    size_t b = 0;
    for (int t = 0; t < RKB_MAX_WORKERS; t++) b += w->bytes[t];
    return b;
}

/* ---- the fan-out -------------------------------------------------------------- */
typedef struct {
    const void *A;        /* [M,K] int8 or fp16 */
    void *C;              /* [M,N] */
    const float *a_scale, *b_scale;
    int out_kind;
} rrun_args;

static int rrun(const rkb_rctx *c, const rkb_rweights *w, int M, const rrun_args *a,
                const char *who)
{
    const int K = w->K, N = w->N;
    const size_t esz = w->kind == RW_F16 ? 2 : w->kind == RW_BF16 ? 4 : 1;
    const size_t osz = a->out_kind == RKB_OUT_F16 ? 2 : 4;
    const int c_dev = rkb_ptr_device(a->C);
    int caller_dev = 0;
    cudaGetDevice(&caller_dev);   /* workers switch devices; the caller's is restored */
    int rows_const = 0;
    if (w->kind == RW_I8_GW || w->kind == RW_I4_GW)
        rows_const = rkb_ptr_device(a->a_scale) < 0 ? rkb_rows_const(a->a_scale, M, K / w->group) : 0;
    int rc = 0;
    int staged = 0;
    for (int t = 0; t < w->nt && !rc; t++) {
        const int n0 = w->n0[t], nsub = w->nsub[t];
        if (nsub <= 0) continue;
        rkb_handle *h = rkb_get(c->fd[t]);
        const void *dA = rkb_stage_in(h, RKB_SCR_A, a->A, (size_t)M * K * esz);
        if (!dA) { rc = ROCKET_E_NOMEM; break; }
        if (dA != a->A) staged = 1;
        /* write straight into C when it lives on this GPU, else into scratch */
        uint8_t *cslice = (uint8_t *)a->C + (size_t)n0 * osz;
        const int direct = (c_dev == h->device) && (((uintptr_t)cslice & 15) == 0);
        void *dC = direct ? (void *)cslice : rkb_scratch(h, RKB_SCR_C, (size_t)M * nsub * osz);
        const long ldc = direct ? N : nsub;
        if (!direct) staged = 1;
        if (!dC) { rc = ROCKET_E_NOMEM; break; }
        switch (w->kind) {
        case RW_F16:
            rc = rkb_dense_on(h, RKB_IN_F16, RKB_OUT_F16, M, nsub, K, dA, K, w->dev[t], K, dC, ldc);
            break;
        case RW_I8:
            rc = rkb_dense_on(h, RKB_IN_I8, RKB_OUT_I32, M, nsub, K, dA, K, w->dev[t], K, dC, ldc);
            break;
        case RW_BF16: {
            void *a16 = rkb_scratch(h, RKB_SCR_AUX, (size_t)M * K * 2);
            rc = a16 ? rkb_f32_to_bf16(dA, (size_t)M * K, a16, h->stream) : ROCKET_E_NOMEM;
            if (!rc) rc = rkb_dense_on(h, RKB_IN_BF16, RKB_OUT_F32, M, nsub, K, a16, K, w->dev[t], K, dC, ldc);
            break;
        }
        case RW_I4: {
            rkb_wgemm_desc d;
            memset(&d, 0, sizeof d);
            d.M = M; d.N = nsub; d.K = K; d.w_bits = 4; d.a_f16 = 0;
            d.A = dA; d.lda = K; d.Wq = w->dev[t]; d.Ws = NULL;
            d.C = dC; d.ldc = ldc; d.out_kind = RKB_OUT_I32;
            rkb_count(0, 1);
            int ps = rkb_prof_begin(h);
            rc = rkb_wgemm_run(&d, h->err_dev, h->stream);
            rkb_prof_end(h, ps, RKB_K_WGEMM_W4_I8);
            break;
        }
        case RW_I8_GW:
        case RW_I4_GW:
            rc = rkb_gw_on(h, M, nsub, K, w->group, w->kind == RW_I8_GW ? 8 : 4, dA, a->a_scale,
                           rows_const, w->dev[t], a->b_scale + (size_t)n0 * (K / w->group), dC, ldc,
                           a->out_kind);
            break;
        }
        if (!rc && !direct) {
            if (cudaMemcpy2DAsync(cslice, (size_t)N * osz, dC, (size_t)nsub * osz, (size_t)nsub * osz,
                                  (size_t)M, cudaMemcpyDefault, h->stream) != cudaSuccess) {
                ROCKET_LOGE("%s: slice copy failed: %s\n", who, cudaGetErrorString(cudaGetLastError()));
                rc = ROCKET_E_DEVICE;
            }
        }
        rkb_count(1, 0);
    }
    /* Deferred completion (rocket_b200_set_async): with every operand already
     * on the workers' GPUs nothing host-visible is pending, so the call can
     * return after the launches; rocket_b200_ctx_sync collects the status. */
    const int gw = (w->kind == RW_I8_GW || w->kind == RW_I4_GW);
    if (!rc && rkb_async_enabled() && !staged && !gw) {
        cudaSetDevice(caller_dev);
        return 0;
    }
    for (int t = 0; t < w->nt; t++) {
        if (w->nsub[t] <= 0) continue;
        int fr = rkb_finish(rkb_get(c->fd[t]), who);
        if (!rc) rc = fr;
    }
    cudaSetDevice(caller_dev);
    return rc;
}

int rocket_b200_ctx_sync(const void *ctx)
{
    const rkb_rctx *c = ctx;
    if (!c) return ROCKET_E_SHAPE;
    int rc = 0, dev0 = 0;
    cudaGetDevice(&dev0);
    for (int t = 0; t < c->nthreads; t++) {
        int fr = rkb_finish(rkb_get(c->fd[t]), "rocket_b200_ctx_sync");
        if (!rc) rc = fr;
    }
    cudaSetDevice(dev0);
    return rc;
}

static int resolve(const rkb_rweights *w, int M, int K, int N, const char *who)
{
    if (M <= 0 || M % 4) {
        ROCKET_LOGE("%s: M=%d must be a positive multiple of 4 -- pad rows caller-side\n", who, M);
        return ROCKET_E_SHAPE;
    }
    if (K != w->K || N != w->N) {
        ROCKET_LOGE("%s: shape K=%d N=%d != packed %d/%d\n", who, K, N, w->K, w->N);
        return ROCKET_E_SHAPE;
    }
    return 0;
}

/* ---- fp16 ----------------------------------------------------------------------- */
rocket_ctx *rocket_ctx_create(int nthreads)
{
    rocket_ctx *c = calloc(1, sizeof *c);
    if (!c) return NULL;
    if (rctx_init(&c->r, nthreads, 16, "rocket_ctx_create")) { free(c); return NULL; }
    return c;
}

void rocket_ctx_free(rocket_ctx *ctx)
{
    if (!ctx) return;
    rctx_free(&ctx->r);
    free(ctx);
}

rocket_weights *rocket_weights_pack(rocket_ctx *ctx, int M, int K, int N, const _Float16 *B)
{
    if (!ctx || !B) return NULL;
    if (rocket_matmul_plan(M, K, N, NULL, NULL, NULL) < 0 || M % 4) {
        ROCKET_LOGE("rocket_weights_pack: bad shape M=%d K=%d N=%d\n", M, K, N);
        return NULL;
    }
    rocket_weights *w = calloc(1, sizeof *w);
    if (!w) return NULL;
    if (rweights_pack(&ctx->r, &w->w, RW_F16, M, K, N, B, 0, "rocket_weights_pack")) { free(w); return NULL; }
    return w;
}

void rocket_weights_free(rocket_ctx *ctx, rocket_weights *w)
{
    if (!ctx || !w) return;
    rweights_free(&ctx->r, &w->w);
    free(w);
}

int rocket_matmul_fp16_prepacked(rocket_ctx *ctx, int M, int K, int N, const _Float16 *A,
                                 _Float16 *C, rocket_weights *w)
{
    if (!ctx || !w || !A || !C) return ROCKET_E_SHAPE;
    int rc = resolve(&w->w, M, K, N, "rocket_matmul_fp16_prepacked");
    if (rc) return rc;
    rrun_args a = { A, C, NULL, NULL, RKB_OUT_F16 };
    return rrun(&ctx->r, &w->w, M, &a, "rocket_matmul_fp16_prepacked");
}

int rocket_matmul_fp16_mt(int M, int K, int N, const _Float16 *A, const _Float16 *B, _Float16 *C,
                          int nthreads)
{
    if (rocket_matmul_plan(M, K, N, NULL, NULL, NULL) < 0 || !A || !B || !C) return ROCKET_E_SHAPE;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > RKB_MAX_WORKERS) nthreads = RKB_MAX_WORKERS;
    rkb_rctx c;
    if (rctx_init(&c, nthreads, 16, "rocket_matmul_fp16_mt")) return ROCKET_E_DEVICE;
    rkb_rweights w;
    int rc = rweights_pack(&c, &w, RW_F16, M, K, N, B, 0, "rocket_matmul_fp16_mt");
    if (!rc) {
        rrun_args a = { A, C, NULL, NULL, RKB_OUT_F16 };
        rc = rrun(&c, &w, M, &a, "rocket_matmul_fp16_mt");
        rweights_free(&c, &w);
    }
    rctx_free(&c);
    return rc;
}

/* ---- int8 ------------------------------------------------------------------------ */
rocket_i8_ctx *rocket_i8_ctx_create(int nthreads)
{
    rocket_i8_ctx *c = calloc(1, sizeof *c);
    if (!c) return NULL;
    if (rctx_init(&c->r, nthreads, 32, "rocket_i8_ctx_create")) { free(c); return NULL; }
    return c;
}

void rocket_i8_ctx_free(rocket_i8_ctx *ctx)
{
    if (!ctx) return;
    rctx_free(&ctx->r);
    free(ctx);
}

static int i8_shape_ok(const char *who, int M, int K, int N)
{
    if (M <= 0 || M % 4 || K <= 0 || K % 32 || N <= 0 || N % 32) {
        ROCKET_LOGE("%s: bad shape M=%d K=%d N=%d (need M%%4, K%%32, N%%32)\n", who, M, K, N);
        return 0;
    }
    return 1;
}

rocket_i8_weights *rocket_i8_weights_pack(rocket_i8_ctx *ctx, int M, int K, int N, const int8_t *B)
{
    if (!ctx || !B || !i8_shape_ok("rocket_i8_weights_pack", M, K, N)) return NULL;
    rocket_i8_weights *w = calloc(1, sizeof *w);
    if (!w) return NULL;
    if (rweights_pack(&ctx->r, &w->w, RW_I8, M, K, N, B, 0, "rocket_i8_weights_pack")) { free(w); return NULL; }
    return w;
}

rocket_i8_weights *rocket_i8_weights_pack_gw(rocket_i8_ctx *ctx, int M, int K, int N,
                                             const int8_t *B, int group)
{
    if (!ctx || !B || !i8_shape_ok("rocket_i8_weights_pack_gw", M, K, N)) return NULL;
    if (group < 32 || group % 32 || K % group) {
        ROCKET_LOGE("rocket_i8_weights_pack_gw: bad group=%d (need >=32, %%32, |K) K=%d\n", group, K);
        return NULL;
    }
    rocket_i8_weights *w = calloc(1, sizeof *w);
    if (!w) return NULL;
    if (rweights_pack(&ctx->r, &w->w, RW_I8_GW, M, K, N, B, group, "rocket_i8_weights_pack_gw")) {
        free(w);
        return NULL;
    }
    return w;
}

void rocket_i8_weights_free(rocket_i8_ctx *ctx, rocket_i8_weights *w)
{
    if (!ctx || !w) return;
    rweights_free(&ctx->r, &w->w);
    free(w);
}

size_t rocket_i8_weights_bytes(const rocket_i8_weights *w) { return w ? rweights_bytes(&w->w) : 0; }

int rocket_matmul_int8_prepacked(rocket_i8_ctx *ctx, int M, int K, int N, const int8_t *A,
                                 int32_t *C, rocket_i8_weights *w)
{
    if (!ctx || !w || !A || !C) return ROCKET_E_SHAPE;
    if (w->w.kind != RW_I8) {
        ROCKET_LOGE("rocket_matmul_int8_prepacked: weight is group-wise -- use rocket_matmul_int8_prepacked_gw\n");
        return ROCKET_E_SHAPE;
    }
    int rc = resolve(&w->w, M, K, N, "rocket_matmul_int8_prepacked");
    if (rc) return rc;
    rrun_args a = { A, C, NULL, NULL, RKB_OUT_I32 };
    return rrun(&ctx->r, &w->w, M, &a, "rocket_matmul_int8_prepacked");
}

int rocket_matmul_int8_prepacked_gw(rocket_i8_ctx *ctx, int M, int K, int N, const int8_t *A,
                                    const float *a_scale, const float *b_scale, float *Cf,
                                    rocket_i8_weights *w)
{
    if (!ctx || !w || !A || !a_scale || !b_scale || !Cf) return ROCKET_E_SHAPE;
    if (w->w.kind != RW_I8_GW) {
        ROCKET_LOGE("rocket_matmul_int8_prepacked_gw: weight is per-channel -- use rocket_matmul_int8_prepacked\n");
        return ROCKET_E_SHAPE;
    }
    int rc = resolve(&w->w, M, K, N, "rocket_matmul_int8_prepacked_gw");
    if (rc) return rc;
    rrun_args a = { A, Cf, a_scale, b_scale, RKB_OUT_F32 };
    return rrun(&ctx->r, &w->w, M, &a, "rocket_matmul_int8_prepacked_gw");
}

/* ---- int4 ------------------------------------------------------------------------ */
rocket_i4_ctx *rocket_i4_ctx_create(int nthreads)
{
    rocket_i4_ctx *c = calloc(1, sizeof *c);
    if (!c) return NULL;
    if (rctx_init(&c->r, nthreads, 64, "rocket_i4_ctx_create")) { free(c); return NULL; }
    return c;
}

void rocket_i4_ctx_free(rocket_i4_ctx *ctx)
{
    if (!ctx) return;
    rctx_free(&ctx->r);
    free(ctx);
}

static int i4_shape_ok(const char *who, int M, int K, int N)
{
    if (M <= 0 || M % 4 || K <= 0 || K % 32 || N <= 0 || N % 64) {
        ROCKET_LOGE("%s: bad shape M=%d K=%d N=%d (need M%%4, K%%32, N%%64)\n", who, M, K, N);
        return 0;
    }
    return 1;
}

rocket_i4_weights *rocket_i4_weights_pack(rocket_i4_ctx *ctx, int M, int K, int N, const int8_t *B)
{
    if (!ctx || !B || !i4_shape_ok("rocket_i4_weights_pack", M, K, N)) return NULL;
    rocket_i4_weights *w = calloc(1, sizeof *w);
    if (!w) return NULL;
    if (rweights_pack(&ctx->r, &w->w, RW_I4, M, K, N, B, 0, "rocket_i4_weights_pack")) { free(w); return NULL; }
    return w;
}

rocket_i4_weights *rocket_i4_weights_pack_gw(rocket_i4_ctx *ctx, int M, int K, int N,
                                             const int8_t *B, int group)
{
    if (!ctx || !B || !i4_shape_ok("rocket_i4_weights_pack_gw", M, K, N)) return NULL;
    if (group < 32 || group % 32 || K % group || 49 * group >= 32767) {
        ROCKET_LOGE("rocket_i4_weights_pack_gw: bad group=%d (need %%32, |K, 49*group<32767)\n", group);
        return NULL;
    }
    rocket_i4_weights *w = calloc(1, sizeof *w);
    if (!w) return NULL;
    if (rweights_pack(&ctx->r, &w->w, RW_I4_GW, M, K, N, B, group, "rocket_i4_weights_pack_gw")) {
        free(w);
        return NULL;
    }
    return w;
}

void rocket_i4_weights_free(rocket_i4_ctx *ctx, rocket_i4_weights *w)
{
    if (!ctx || !w) return;
    rweights_free(&ctx->r, &w->w);
    free(w);
}

size_t rocket_i4_weights_bytes(const rocket_i4_weights *w) { return w ? rweights_bytes(&w->w) : 0; }

int rocket_matmul_int4_prepacked(rocket_i4_ctx *ctx, int M, int K, int N, const int8_t *A,
                                 int32_t *C, rocket_i4_weights *w)
{
    if (!ctx || !w || !A || !C) return ROCKET_E_SHAPE;
    if (w->w.kind != RW_I4) {
        ROCKET_LOGE("rocket_matmul_int4_prepacked: weight is group-wise -- use rocket_matmul_int4_prepacked_gw\n");
        return ROCKET_E_SHAPE;
    }
    int rc = resolve(&w->w, M, K, N, "rocket_matmul_int4_prepacked");
    if (rc) return rc;
    rrun_args a = { A, C, NULL, NULL, RKB_OUT_I32 };
    return rrun(&ctx->r, &w->w, M, &a, "rocket_matmul_int4_prepacked");
}

int rocket_matmul_int4_prepacked_gw(rocket_i4_ctx *ctx, int M, int K, int N, const int8_t *A,
                                    const float *a_scale, const float *b_scale, float *Cf,
                                    rocket_i4_weights *w)
{
    if (!ctx || !w || !A || !a_scale || !b_scale || !Cf) return ROCKET_E_SHAPE;
    if (w->w.kind != RW_I4_GW) {
        ROCKET_LOGE("rocket_matmul_int4_prepacked_gw: weight is per-channel -- use rocket_matmul_int4_prepacked\n");
        return ROCKET_E_SHAPE;
    }
    int rc = resolve(&w->w, M, K, N, "rocket_matmul_int4_prepacked_gw");
    if (rc) return rc;
    rrun_args a = { A, Cf, a_scale, b_scale, RKB_OUT_F32 };
    return rrun(&ctx->r, &w->w, M, &a, "rocket_matmul_int4_prepacked_gw");
}

/* ---- streaming contexts: weights re-uploaded every call ----------------------
 * Reference: src/rocket_prepacked.c:459-505 (rocket_stream / _fused) and
 * src/rocket_bf16_stream.c:344-549 (bf16 mt / stream).  A stream keeps its
 * workers and their weight buffers across calls and re-fills them with each
 * call's B (or the N-concatenation of several Bs), so an LLM's repeating shape
 * set pays device allocation once. */
struct rocket_stream      { rkb_rctx r; rkb_rweights w; };
struct rocket_bf16_stream { rkb_rctx r; rkb_rweights w; };

rocket_stream *rocket_stream_create(int nthreads)
{
    rocket_stream *s = calloc(1, sizeof *s);
    if (!s) return NULL;
    if (rctx_init(&s->r, nthreads, 16, "rocket_stream_create")) { free(s); return NULL; }
    return s;
}

void rocket_stream_free(rocket_stream *s)
{
    if (!s) return;
    rweights_free(&s->r, &s->w);
    rctx_free(&s->r);
    free(s);
}

int rocket_matmul_fp16_stream_fused(rocket_stream *s, int M, int K, const _Float16 *const *Bs,
                                    const int *Ns, int nseg, const _Float16 *A, _Float16 *C)
{
    const char *who = "rocket_matmul_fp16_stream_fused";
    if (!s || !Bs || !Ns || !A || !C || nseg < 1 || nseg > ROCKET_MAX_FUSE) return ROCKET_E_SHAPE;
    int N = 0;
    for (int i = 0; i < nseg; i++) {
        if (!Bs[i] || Ns[i] <= 0) return ROCKET_E_SHAPE;
        N += Ns[i];
    }
    if (rocket_matmul_plan(M, K, N, NULL, NULL, NULL) < 0) return ROCKET_E_SHAPE;
    int rc = rweights_fill(&s->r, &s->w, RW_F16, M, K, N, nseg, (const void *const *)Bs, Ns, 0, 0, who);
    if (rc) return rc;
    rrun_args a = { A, C, NULL, NULL, RKB_OUT_F16 };
    return rrun(&s->r, &s->w, M, &a, who);
}

int rocket_matmul_fp16_stream(rocket_stream *s, int M, int K, int N, const _Float16 *A,
                              const _Float16 *B, _Float16 *C)
{
    const _Float16 *bs[1] = {B};
    const int ns[1] = {N};
    return rocket_matmul_fp16_stream_fused(s, M, K, bs, ns, 1, A, C);
}

rocket_bf16_stream *rocket_bf16_stream_create(int nthreads)
{
    rocket_bf16_stream *s = calloc(1, sizeof *s);
    if (!s) return NULL;
    if (rctx_init(&s->r, nthreads, 16, "rocket_bf16_stream_create")) { free(s); return NULL; }
    return s;
}

void rocket_bf16_stream_free(rocket_bf16_stream *s)
{
    if (!s) return;
    rweights_free(&s->r, &s->w);
    rctx_free(&s->r);
    free(s);
}

int rocket_matmul_bf16_stream(rocket_bf16_stream *s, int M, int K, int N, const float *A,
                              const float *B, float *C)
{
    const char *who = "rocket_matmul_bf16_stream";
    if (!s || !A || !B || !C || rocket_matmul_plan(M, K, N, NULL, NULL, NULL) < 0) return ROCKET_E_SHAPE;
    const void *bs[1] = {B};
    const int ns[1] = {N};
    int rc = rweights_fill(&s->r, &s->w, RW_BF16, M, K, N, 1, bs, ns, 0, 0, who);
    if (rc) return rc;
    rrun_args a = { A, C, NULL, NULL, RKB_OUT_F32 };
    return rrun(&s->r, &s->w, M, &a, who);
}

int rocket_matmul_bf16_mt(int M, int K, int N, const float *A, const float *B, float *C, int nthreads)
{
    rocket_bf16_stream *s = rocket_bf16_stream_create(nthreads);
    if (!s) return ROCKET_E_DEVICE;
    int rc = rocket_matmul_bf16_stream(s, M, K, N, A, B, C);
    rocket_bf16_stream_free(s);
    return rc;
}
