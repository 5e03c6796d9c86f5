/*
 * rocket_matmul.c -- tiling previews and the one-shot matmul entry points.
 *
 * Reference: src/rocket_matmul.c (plans :498-568, :2383-2437, :2671-2714,
 * :2917; fp16 :1945-1998; int8 :2439-2627; int8 group-wise :2716-2871; int4
 * :2958-3114; int4 group-wise :3132-3282).  The reference tiles each call into
 * <=256x256 NPU programs, packs A/B into cube layouts, submits, waits and
 * accumulates K-partials on the host.  Here a call stages host operands into
 * device scratch (device operands are used in place), launches one persistent
 * tcgen05 kernel, copies C back and waits -- synchronous like the reference.
 */
#include <stdlib.h>
#include <string.h>

#include "rocket_matmul.h"
#include "rocket_b200.h"
#include "rocket_hw_profile.h"
#include "rkb_internal.h"

/* ---- shape rules (reference API.md:96-104) ------------------------------ */
static int m_ok(int M, int allow_one) { return M > 0 && (M % 4 == 0 || (allow_one && M == 1)); }

static int plan_common(int M, int K, int N, int kt, int *Mt, int *Kt, int *Nt)
{
    if (Mt) *Mt = M < 128 ? M : 128;
    if (Kt) *Kt = K < kt ? K : kt;
    if (Nt) *Nt = N < 256 ? N : 256;
    long tiles = (long)((M + 127) / 128) * ((N + 255) / 256);
    return tiles > 0x7fffffff ? 0x7fffffff : (int)tiles;
}

int rocket_matmul_plan(int M, int K, int N, int *Mt, int *Kt, int *Nt)
{
    if (!m_ok(M, 1) || K <= 0 || N <= 0 || K % 32 || N % 16) return ROCKET_E_SHAPE;
    return plan_common(M, K, N, 64, Mt, Kt, Nt);
}

int rocket_matmul_plan_int8(int M, int K, int N, int *Mt, int *Kt, int *Nt)
{
    if (!m_ok(M, 1) || K <= 0 || N <= 0 || K % 32 || N % 32) return ROCKET_E_SHAPE;
    return plan_common(M, K, N, 128, Mt, Kt, Nt);
}

static int gw_group_ok(int K, int group) { return group >= 32 && group % 32 == 0 && K % group == 0; }

int rocket_matmul_plan_int8_gw(int M, int K, int N, int group, int *Mt, int *Kt, int *Nt)
{
    if (!m_ok(M, 0) || K <= 0 || N <= 0 || K % 32 || N % 32 || !gw_group_ok(K, group))
        return ROCKET_E_SHAPE;
    /* Kt = K per exact integer partial of the precise kernel: the group
     * (int32 partials are exact for any group) */
    return plan_common(M, K, N, group, Mt, Kt, Nt);
}

/* ---- hardware profile (reference include/rocket_hw_profile.h:60-108) ----- */
static const struct rocket_hw_profile g_hw_b200 = {
    "b200", 0, 0, 256, 16, 8, 16, ~0u, NULL, 1,
};

const struct rocket_hw_profile *rocket_hw_current(void) { return &g_hw_b200; }

const struct rocket_hw_profile *rocket_hw_by_name(const char *name)
{
    return name && strcmp(name, "b200") == 0 ? &g_hw_b200 : NULL;
}

int rocket_matmul_plan_int4(int M, int K, int N, int *Mt, int *Kt, int *Nt)
{
    if (!m_ok(M, 1) || K <= 0 || N <= 0 || K % 32 || N % 64) return ROCKET_E_SHAPE;
    return plan_common(M, K, N, 128, Mt, Kt, Nt);
}

/* ---- shared compute helpers -------------------------------------------- */
int rkb_dense_on(rkb_handle *h, int in_kind, int out_kind, int M, int N, int K,
                 const void *dA, long lda, const void *dB, long ldb, void *dC, long ldc)
{
    rkb_gemm_desc d;
    memset(&d, 0, sizeof d);
    d.in_kind = in_kind; d.out_kind = out_kind;
    d.M = M; d.N = N; d.K = K;
    d.A = dA; d.lda = lda; d.B = dB; d.ldb = ldb; d.C = dC; d.ldc = ldc;
    const size_t wb = rkb_gemm_workspace_bytes(&d);
    if (wb && !(d.workspace = rkb_scratch(h, RKB_SCR_SPLIT, wb))) return ROCKET_E_NOMEM;
    rkb_count(0, rkb_gemm_launches(&d));
    int ps = rkb_prof_begin(h);
    int rc = rkb_gemm_run(&d, h->err_dev, h->stream);
    rkb_prof_end(h, ps, in_kind == RKB_IN_F16 ? RKB_K_GEMM_F16 : RKB_K_GEMM_I8);
    return rc;
}

int rkb_rows_const(const float *a_scale, int M, int nG)
{
    for (int m = 0; m < M; m++) {
        const float *r = a_scale + (size_t)m * nG;
        for (int g = 1; g < nG; g++)
            if (r[g] != r[0]) return 0;
    }
    return 1;
}

/* Group-wise mode for this process: 0 precise (default), 1 fast.  The
 * environment variable ROCKET_GW_FAST=1 selects the fast mode too. */
static int g_gw_mode = -1;

int rocket_b200_gw_mode(int mode)
{
    if (mode < 0 || mode > 1) return ROCKET_E_SHAPE;
    __atomic_store_n(&g_gw_mode, mode, __ATOMIC_RELAXED);
    return 0;
}

static int gw_fast(void)
{
    int m = __atomic_load_n(&g_gw_mode, __ATOMIC_RELAXED);
    if (m < 0) m = rkb_env_long("ROCKET_GW_FAST", 0) ? 1 : 0;
    return m == 1;
}

/* Precise form (the reference's definition, src/rocket_matmul.c:2842-2856):
 * exact integer partials per group from the fp16 MMA on unscaled operands,
 * scaled and summed across groups in fp32 by the kernel's epilogue. */
static int gw_precise_on(rkb_handle *h, int M, int N, int K, int group, int w_bits,
                         const int8_t *dA, const float *das, int a_rows_const,
                         const void *dWq, const float *dbs, void *dC, long ldc, int out_kind)
{
    const int nG = K / group;
    float *sc = rkb_scratch(h, RKB_SCR_ROW, (size_t)M * (a_rows_const ? 1 : nG) * sizeof(float));
    if (!sc) return ROCKET_E_NOMEM;
    int ps = rkb_prof_begin(h);
    int rc = a_rows_const ? rkb_gather_row_scale(das, M, nG, sc, h->stream)
                          : rkb_scale_transpose(das, M, nG, sc, h->stream);
    rkb_prof_end(h, ps, RKB_K_PRESCALE);
    if (rc) return rc;
    rkb_wgemm_desc d;
    memset(&d, 0, sizeof d);
    d.M = M; d.N = N; d.K = K;
    d.w_bits = w_bits;
    d.A = dA; d.lda = K;                    /* int8 activations as given */
    d.Wq = dWq;
    d.C = dC; d.ldc = ldc; d.out_kind = out_kind;
    d.row_scale = a_rows_const ? sc : NULL;
    d.a_scale_t = a_rows_const ? NULL : sc;
    d.b_scale = dbs;
    d.group = group;
    rkb_count(0, 2);
    ps = rkb_prof_begin(h);
    rc = rkb_wgemm_xi_run(&d, h->err_dev, h->stream);
    rkb_prof_end(h, ps, RKB_K_WGEMM_GW_I8);
    return rc;
}

int rkb_gw_on(rkb_handle *h, int M, int N, int K, int group, int w_bits,
              const int8_t *dA, const float *a_scale, int a_rows_const,
              const void *dWq, const float *b_scale, void *dC, long ldc, int out_kind)
{
    const int nG = K / group;
    const float *dbs = rkb_stage_in(h, RKB_SCR_BS, b_scale, (size_t)N * nG * sizeof(float));
    const float *das = rkb_stage_in(h, RKB_SCR_AS, a_scale, (size_t)M * nG * sizeof(float));
    if (!dbs || !das) return ROCKET_E_NOMEM;
    if (!gw_fast())
        return gw_precise_on(h, M, N, K, group, w_bits, dA, das, a_rows_const, dWq, dbs, dC, ldc,
                             out_kind);
    /* fast form: w * b_scale (and a * a_scale when it varies with g) rounded to
     * fp16 once, fp32 accumulation (about 3e-4 relative) */
    void *ws = rkb_scratch(h, RKB_SCR_WS, rkb_wpack_scales_bytes(N, K));
    void *af = rkb_scratch(h, RKB_SCR_AUX, (size_t)M * K * 2);
    if (!ws || !af) return ROCKET_E_NOMEM;
    int ps = rkb_prof_begin(h);
    int rc = rkb_wpack_scales(dbs, N, K, group, ws, h->stream);
    rkb_prof_end(h, ps, RKB_K_PACK);
    float *row = NULL;
    ps = rkb_prof_begin(h);
    if (!rc && a_rows_const) {
        row = rkb_scratch(h, RKB_SCR_ROW, (size_t)M * sizeof(float));
        if (!row) return ROCKET_E_NOMEM;
        rc = rkb_gather_row_scale(das, M, nG, row, h->stream);
        if (!rc) rc = rkb_prescale_a(dA, NULL, M, K, group, af, h->stream);
    } else if (!rc) {
        rc = rkb_prescale_a(dA, das, M, K, group, af, h->stream);
    }
    rkb_prof_end(h, ps, RKB_K_PRESCALE);
    if (rc) return rc;
    rkb_wgemm_desc d;
    memset(&d, 0, sizeof d);
    d.M = M; d.N = N; d.K = K;
    d.w_bits = w_bits; d.a_f16 = 1;
    d.A = af; d.lda = K;
    d.Wq = dWq; d.Ws = ws;
    d.C = dC; d.ldc = ldc; d.out_kind = out_kind;
    d.row_scale = row;
    rkb_count(0, a_rows_const ? 4 : 3);
    ps = rkb_prof_begin(h);
    rc = rkb_wgemm_run(&d, h->err_dev, h->stream);
    rkb_prof_end(h, ps, w_bits == 4 ? RKB_K_WGEMM_W4_F16 : RKB_K_WGEMM_W8_F16);
    return rc;
}

/* ---- one-shot entries ---------------------------------------------------- */
int rkb_oneshot_dense(const char *who, int fd, int in_kind, int out_kind, int M, int K, int N,
                      const void *A, const void *B, void *C, int finish)
{
    rkb_handle *h = rkb_get(fd);
    if (!h) {
        ROCKET_LOGE("%s: bad device handle %d\n", who, fd);
        return ROCKET_E_DEVICE;
    }
    if (!A || !B || !C) return ROCKET_E_SHAPE;
    const size_t esz = in_kind == RKB_IN_I8 ? 1 : in_kind == RKB_IN_TF32 ? 4 : 2;
    const size_t osz = out_kind == RKB_OUT_F16 ? 2 : 4;
    const void *dA = rkb_stage_in(h, RKB_SCR_A, A, (size_t)M * K * esz);
    const void *dB = rkb_stage_in(h, RKB_SCR_B, B, (size_t)N * K * esz);
    int cb = 0;
    void *dC = rkb_stage_out(h, RKB_SCR_C, C, (size_t)M * N * osz, &cb);
    if (!dA || !dB || !dC) return ROCKET_E_NOMEM;
    int rc = rkb_dense_on(h, in_kind, out_kind, M, N, K, dA, K, dB, K, dC, N);
    if (!rc) rc = rkb_stage_out_finish(h, C, dC, (size_t)M * N * osz, cb);
    rkb_count(1, 0);
    if (!finish && !rc) return 0;   /* caller waits once for a batch of calls */
    if (!rc && rkb_async_enabled() && dA == A && dB == B && !cb) return 0;   /* deferred */
    int fr = rkb_finish(h, who);
    return rc ? rc : fr;
}

static int oneshot_dense(const char *who, int fd, int in_kind, int out_kind, int M, int K, int N,
                         const void *A, const void *B, void *C)
{
    return rkb_oneshot_dense(who, fd, in_kind, out_kind, M, K, N, A, B, C, 1);
}

int rocket_matmul_fp16(int fd, int M, int K, int N, const _Float16 *A, const _Float16 *B,
                       _Float16 *C)
{
    if (rocket_matmul_plan(M, K, N, NULL, NULL, NULL) < 0) {
        ROCKET_LOGE("rocket_matmul_fp16: bad shape M=%d K=%d N=%d (need M%%4|M==1, K%%32, N%%16)\n", M, K, N);
        return ROCKET_E_SHAPE;
    }
    return oneshot_dense("rocket_matmul_fp16", fd, RKB_IN_F16, RKB_OUT_F16, M, K, N, A, B, C);
}

int rocket_matmul_int8(int fd, int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C)
{
    if (rocket_matmul_plan_int8(M, K, N, NULL, NULL, NULL) < 0) {
        ROCKET_LOGE("rocket_matmul_int8: bad shape M=%d K=%d N=%d (need M%%4|M==1, K%%32, N%%32)\n", M, K, N);
        return ROCKET_E_SHAPE;
    }
    return oneshot_dense("rocket_matmul_int8", fd, RKB_IN_I8, RKB_OUT_I32, M, K, N, A, B, C);
}

int rocket_matmul_int4_ex(int fd, int M, int K, int N, const int8_t *A, const int8_t *B,
                          int32_t *C, int kt_cap)
{
    (void)kt_cap;   /* int32 accumulation never saturates; the cap has nothing to bound */
    if (rocket_matmul_plan_int4(M, K, N, NULL, NULL, NULL) < 0) {
        ROCKET_LOGE("rocket_matmul_int4: bad shape M=%d K=%d N=%d (need M%%4|M==1, K%%32, N%%64)\n", M, K, N);
        return ROCKET_E_SHAPE;
    }
    /* one value per int8_t: the int8 kernel contracts them exactly */
    return oneshot_dense("rocket_matmul_int4", fd, RKB_IN_I8, RKB_OUT_I32, M, K, N, A, B, C);
}

int rocket_matmul_int4(int fd, int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C)
{
    return rocket_matmul_int4_ex(fd, M, K, N, A, B, C, 0);
}

static int oneshot_gw(const char *who, int fd, int w_bits, int M, int K, int N, const int8_t *A,
                      const int8_t *B, const float *a_scale, const float *b_scale, float *Cf,
                      int group)
{
    rkb_handle *h = rkb_get(fd);
    if (!h) {
        ROCKET_LOGE("%s: bad device handle %d\n", who, fd);
        return ROCKET_E_DEVICE;
    }
    if (!A || !B || !a_scale || !b_scale || !Cf) return ROCKET_E_SHAPE;
    const int nG = K / group;
    const int8_t *dA = rkb_stage_in(h, RKB_SCR_A, A, (size_t)M * K);
    const int8_t *dB = rkb_stage_in(h, RKB_SCR_B, B, (size_t)N * K);
    void *wq = rkb_scratch(h, RKB_SCR_WQ, rkb_wpack_codes_bytes(N, K, w_bits));
    int cb = 0;
    void *dC = rkb_stage_out(h, RKB_SCR_C, Cf, (size_t)M * N * sizeof(float), &cb);
    if (!dA || !dB || !wq || !dC) return ROCKET_E_NOMEM;
    int rows_const = rkb_ptr_device(a_scale) < 0 ? rkb_rows_const(a_scale, M, nG) : 0;
    int ps = rkb_prof_begin(h);
    int rc = rkb_wpack_codes(dB, N, K, w_bits, wq, h->stream);
    rkb_prof_end(h, ps, RKB_K_PACK);
    if (!rc) rc = rkb_gw_on(h, M, N, K, group, w_bits, dA, a_scale, rows_const, wq, b_scale, dC, N,
                            RKB_OUT_F32);
    if (!rc) rc = rkb_stage_out_finish(h, Cf, dC, (size_t)M * N * sizeof(float), cb);
    rkb_count(1, 1);
    int fr = rkb_finish(h, who);
    return rc ? rc : fr;
}

int rocket_matmul_int8_groupwise(int fd, int M, int K, int N, const int8_t *A, const int8_t *B,
                                 const float *a_scale, const float *b_scale, float *Cf, int group)
{
    if (rocket_matmul_plan_int8_gw(M, K, N, group, NULL, NULL, NULL) < 0) {
        ROCKET_LOGE("rocket_matmul_int8_groupwise: bad shape M=%d K=%d N=%d group=%d\n", M, K, N, group);
        return ROCKET_E_SHAPE;
    }
    return oneshot_gw("rocket_matmul_int8_groupwise", fd, 8, M, K, N, A, B, a_scale, b_scale, Cf, group);
}

int rocket_matmul_int4_groupwise(int fd, int M, int K, int N, const int8_t *A, const int8_t *B,
                                 const float *a_scale, const float *b_scale, float *Cf, int group)
{
    if (!m_ok(M, 0) || K <= 0 || N <= 0 || K % 32 || N % 64 || !gw_group_ok(K, group) ||
        49 * group >= 32767) {
        ROCKET_LOGE("rocket_matmul_int4_groupwise: bad shape M=%d K=%d N=%d group=%d\n", M, K, N, group);
        return ROCKET_E_SHAPE;
    }
    return oneshot_gw("rocket_matmul_int4_groupwise", fd, 4, M, K, N, A, B, a_scale, b_scale, Cf, group);
}
