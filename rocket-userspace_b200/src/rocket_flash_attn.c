/*
 * rocket_flash_attn.c -- masked grouped-query attention entries (reference
 * include/rocket_attn.h:46-150, src/rocket_attn.c:700-900).
 *
 * The reference runs per-head QK and AV matmuls on the NPU and the mask and
 * softmax on the host.  Here one fused kernel (csrc/fa_tc.cu) computes every
 * head: the score matrix never leaves the SM.
 *   _mt   runs the same kernel; the reference spread heads over worker fds
 *         because per-head work was dispatch-bound, which one launch over all
 *         heads already removes.  Results are identical to the single entry.
 *   _ctx  keeps a handle open across calls (one per process-lifetime context).
 * The reference's fd < 0 host-reference mode is not offered.
 */
#include <stdlib.h>
#include <string.h>

#include "rocket_attn.h"
#include "rkb_internal.h"

static int fa_run(int fd, int T, int n_kv, int dh, int dv, int nh, int nkvh, float scale, float softcap,
                  const _Float16 *Q, const _Float16 *K, const _Float16 *V, const _Float16 *mask,
                  _Float16 *out, const char *who)
{
    if (T < 1 || n_kv < 1 || dh < 1 || dv < 1 || nh < 1 || nkvh < 1 || nh % nkvh || dh % 32 || dv % 16 ||
        !Q || !K || !V || !out)
        return ROCKET_E_SHAPE;
    if (dh > 256 || dv > 256) {
        ROCKET_LOGE("%s: head_dim %d / dv %d above 256 not supported\n", who, dh, dv);
        return ROCKET_E_UNSUPPORTED;
    }
    rkb_call c;
    int rc = rkb_call_begin(&c, fd, who);
    if (rc) return rc;
    const size_t qb = (size_t)nh * T * dh * 2, kb = (size_t)nkvh * n_kv * dh * 2;
    const void *dQ = rkb_call_in(&c, Q, qb);
    const void *dK = rkb_call_in(&c, K, kb);
    const void *dM = mask ? rkb_call_in(&c, mask, (size_t)T * n_kv * 2) : NULL;
    /* V rows feed TMA, which needs 16-byte row pitch: re-pitch when n_kv % 8 */
    const long ldv = (n_kv + 7) & ~7;
    const void *dV;
    if (ldv == n_kv) {
        dV = rkb_call_in(&c, V, (size_t)nkvh * dv * n_kv * 2);
    } else {
        void *t = rkb_call_tmp(&c, (size_t)nkvh * dv * ldv * 2);
        if (rkb_ptr_device(V) < 0) c.host_in = 1;
        if (t && cudaMemcpy2DAsync(t, (size_t)ldv * 2, V, (size_t)n_kv * 2, (size_t)n_kv * 2,
                                   (size_t)nkvh * dv, cudaMemcpyDefault, c.h->stream) != cudaSuccess) {
            cudaGetLastError();
            c.rc = ROCKET_E_DEVICE;
        }
        dV = t;
    }
    void *dO = rkb_call_out(&c, out, (size_t)nh * T * dv * 2);
    if (!c.rc) {
        int ps = rkb_prof_begin(c.h);
        rkb_call_check(&c, rkb_flash_attn(dQ, dK, dV, ldv, dM, dO, T, n_kv, dh, dv, nh, nkvh, scale,
                                          softcap, c.h->err_dev, c.h->stream));
        rkb_prof_end(c.h, ps, RKB_K_ATTN);
        rkb_count(0, 1);
    }
    return rkb_call_end(&c);
}

int rocket_flash_attn_fp16(int fd, int n_tokens, int n_kv, int head_dim, int dv, int n_head,
                           int n_kv_heads, float scale, float softcap, const _Float16 *Q,
                           const _Float16 *K, const _Float16 *V, const _Float16 *mask, _Float16 *out)
{
    return fa_run(fd, n_tokens, n_kv, head_dim, dv, n_head, n_kv_heads, scale, softcap, Q, K, V, mask,
                  out, "rocket_flash_attn_fp16");
}

int rocket_flash_attn_fp16_mt(int fd, int n_tokens, int n_kv, int head_dim, int dv, int n_head,
                              int n_kv_heads, float scale, float softcap, const _Float16 *Q,
                              const _Float16 *K, const _Float16 *V, const _Float16 *mask,
                              _Float16 *out, int nthreads)
{
    (void)nthreads;
    int own = -1;
    if (fd < 0 || !rkb_get(fd)) {
        own = rocket_open();
        if (own < 0) return ROCKET_E_DEVICE;
        fd = own;
    }
    int rc = fa_run(fd, n_tokens, n_kv, head_dim, dv, n_head, n_kv_heads, scale, softcap, Q, K, V, mask,
                    out, "rocket_flash_attn_fp16_mt");
    if (own >= 0) rocket_close(own);
    return rc;
}

struct rocket_fa_ctx { int fd; };

rocket_fa_ctx *rocket_fa_ctx_create(int nthreads)
{
    (void)nthreads;
    rocket_fa_ctx *c = calloc(1, sizeof *c);
    if (!c) return NULL;
    c->fd = rocket_open();
    if (c->fd < 0) { free(c); return NULL; }
    return c;
}

void rocket_fa_ctx_free(rocket_fa_ctx *c)
{
    if (!c) return;
    rocket_close(c->fd);
    free(c);
}

int rocket_flash_attn_fp16_ctx(rocket_fa_ctx *c, int n_tokens, int n_kv, int head_dim, int dv, int n_head,
                               int n_kv_heads, float scale, float softcap, const _Float16 *Q,
                               const _Float16 *K, const _Float16 *V, const _Float16 *mask, _Float16 *out)
{
    if (!c) return ROCKET_E_SHAPE;
    return fa_run(c->fd, n_tokens, n_kv, head_dim, dv, n_head, n_kv_heads, scale, softcap, Q, K, V, mask,
                  out, "rocket_flash_attn_fp16_ctx");
}
