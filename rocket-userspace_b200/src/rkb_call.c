/*
 * rkb_call.c -- per-call plumbing shared by the composite entry points (the
 * encoder ops, batched / streaming matmuls, bf16 / int16 / tf32 forms):
 * temporaries from CUDA's stream-ordered allocator (pooled after the first
 * call), staging of caller inputs that are host memory or misaligned,
 * copy-back of outputs, and the closing bounded wait.
 */
#include <stdint.h>
#include <string.h>

#include "rkb_internal.h"



int rkb_call_begin(rkb_call *c, int fd, const char *who)
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

void *rkb_call_tmp(rkb_call *c, size_t bytes)
{
    if (c->rc || c->ntmp >= RKB_CALL_MAX_TMP) { if (!c->rc) c->rc = ROCKET_E_NOMEM; return NULL; }
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
const void *rkb_call_in(rkb_call *c, const void *user, size_t bytes)
{
    if (!user || c->rc) return NULL;
    const int dev = rkb_ptr_device(user);
    if (dev == c->h->device && ((uintptr_t)user & 15) == 0) return user;
    if (dev < 0) c->host_in = 1;
    void *d = rkb_call_tmp(c, bytes);
    if (d && cudaMemcpyAsync(d, user, bytes, cudaMemcpyDefault, c->h->stream) != cudaSuccess) {
        cudaGetLastError();
        c->rc = ROCKET_E_DEVICE;
    }
    return d;
}

/* device buffer for a caller output; copied back in rkb_call_end when needed */
void *rkb_call_out(rkb_call *c, void *user, size_t bytes)
{
    if (c->rc) return NULL;
    if (rkb_ptr_device(user) == c->h->device && ((uintptr_t)user & 15) == 0) return user;
    void *d = rkb_call_tmp(c, bytes);
    if (d && c->nouts < 4) {
        c->outs[c->nouts].user = user;
        c->outs[c->nouts].dev = d;
        c->outs[c->nouts].bytes = bytes;
        c->nouts++;
    }
    return d;
}

void rkb_call_check(rkb_call *c, int rc)
{
    if (!c->rc && rc) c->rc = rc;
}

int rkb_call_end(rkb_call *c)
{
    for (int i = 0; i < c->nouts && !c->rc; i++)
        if (cudaMemcpyAsync(c->outs[i].user, c->outs[i].dev, c->outs[i].bytes, cudaMemcpyDefault,
                            c->h->stream) != cudaSuccess) {
            cudaGetLastError();
            c->rc = ROCKET_E_DEVICE;
        }
    for (int i = 0; i < c->ntmp; i++) cudaFreeAsync(c->tmp[i], c->h->stream);
    rkb_count(1, 0);
    /* rocket_b200_set_async: with every input and output in device memory the
     * call returns after the launches; rocket_b200_sync collects the status */
    if (!c->rc && rkb_async_enabled() && !c->host_in && c->nouts == 0) return 0;
    int fr = rkb_finish(c->h, c->who);
    return c->rc ? c->rc : fr;
}

/* GEMM with fp16 output and fused epilogue: C = act(A W^T + bias) + residual */
void rkb_call_gemm(rkb_call *c, int M, int N, int K, const void *A, long lda, const void *W,
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
    if (wb && !(d.workspace = rkb_call_tmp(c, wb))) return;
    rkb_count(0, rkb_gemm_launches(&d));
    int ps = rkb_prof_begin(c->h);
    rkb_call_check(c, rkb_gemm_run(&d, c->h->err_dev, c->h->stream));
    rkb_prof_end(c->h, ps, RKB_K_GEMM_F16);
}


void rkb_call_gemm_kind(rkb_call *c, int in_kind, int out_kind, int M, int N, int K, const void *A,
                        long lda, const void *B, long ldb, void *C, long ldc)
{
    if (c->rc) return;
    rkb_gemm_desc d;
    memset(&d, 0, sizeof d);
    d.in_kind = in_kind; d.out_kind = out_kind;
    d.M = M; d.N = N; d.K = K;
    d.A = A; d.lda = lda; d.B = B; d.ldb = ldb; d.C = C; d.ldc = ldc;
    const size_t wb = rkb_gemm_workspace_bytes(&d);
    if (wb && !(d.workspace = rkb_call_tmp(c, wb))) return;
    rkb_count(0, rkb_gemm_launches(&d));
    int ps = rkb_prof_begin(c->h);
    rkb_call_check(c, rkb_gemm_run(&d, c->h->err_dev, c->h->stream));
    rkb_prof_end(c->h, ps, in_kind == RKB_IN_I8 ? RKB_K_GEMM_I8 : RKB_K_GEMM_F16);
}
