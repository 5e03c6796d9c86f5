/*
 * rkb_internal.h -- host-side internals of the B200 build of librocketnpu:
 * device handles, scratch pools, pointer staging and the synchronous
 * completion wait every entry point ends with.
 */
#ifndef RKB_INTERNAL_H
#define RKB_INTERNAL_H

#include <stddef.h>
#include <stdint.h>
#include <pthread.h>
#include <cuda_runtime_api.h>

#include "rocket_npu.h"
#include "rocket_log.h"
#include "rkb_kernels.h"

#define RKB_MAX_HANDLES 256
#define RKB_MAX_BOS     1024
#define RKB_MAX_WORKERS 8

enum rkb_scratch_slot {
    RKB_SCR_A = 0, RKB_SCR_B, RKB_SCR_C, RKB_SCR_AS, RKB_SCR_BS, RKB_SCR_AUX,
    RKB_SCR_ROW, RKB_SCR_WQ, RKB_SCR_WS, RKB_SCR_SPLIT, RKB_NSCR
};

/* Kernel families timed by the profiler (rocket_b200_profile_*). */
enum rkb_kfam {
    RKB_K_GEMM_I8 = 0, RKB_K_GEMM_F16, RKB_K_WGEMM_W4_F16, RKB_K_WGEMM_W8_F16, RKB_K_WGEMM_W4_I8,
    RKB_K_PACK, RKB_K_PRESCALE, RKB_K_NORM, RKB_K_SOFTMAX, RKB_K_ATTN, RKB_K_ELEMWISE,
    RKB_K_WGEMM_GW_I8, RKB_NKFAM
};
#define RKB_PROF_SLOTS 4096

typedef struct rkb_handle {
    int in_use;
    int device;
    cudaStream_t stream;
    int *err_host;      /* mapped pinned error word: kernels record bounded-wait expiry */
    int *err_dev;
    void *scr[RKB_NSCR];
    size_t scr_cap[RKB_NSCR];
    struct { void *dptr; void *hptr; size_t size; int live; } bo[RKB_MAX_BOS];
    /* pinned bounce buffers for small pageable host operands (grow-only), the
     * event after each one's last copy, and host copies-out that complete in
     * rkb_finish */
    void *pin[RKB_NSCR + 1];
    size_t pin_cap[RKB_NSCR + 1];
    cudaEvent_t pin_ev[RKB_NSCR + 1];
    struct { void *user; const void *pin; size_t bytes; } pend;
    int npend;
    /* profiler: event pairs recorded around launches, drained in rkb_finish */
    cudaEvent_t ev[RKB_PROF_SLOTS][2];
    int ev_fam[RKB_PROF_SLOTS];
    int ev_used, ev_made;
} rkb_handle;

/* Handle table. */
int          rkb_open_on(int device);           /* fd >= 0 or rocket_status */
rkb_handle  *rkb_get(int fd);                   /* NULL if fd is not open */
int          rkb_device_count(void);

/* Grow-only per-handle device scratch.  NULL on allocation failure. */
void *rkb_scratch(rkb_handle *h, int slot, size_t bytes);

/* Pointer classes. */
int rkb_ptr_device(const void *p);  /* CUDA device owning p, or -1 for host memory */

/* Input staging: returns a device pointer holding `bytes` of `user`.  Device
 * pointers on the handle's device are returned as-is; host or other-device
 * memory is copied (async, on the handle's stream) into scratch `slot`. */
const void *rkb_stage_in(rkb_handle *h, int slot, const void *user, size_t bytes);
/* Output staging: returns the device buffer the kernel should write; when it is
 * scratch, rkb_stage_out_finish copies it back to `user`. */
void *rkb_stage_out(rkb_handle *h, int slot, void *user, size_t bytes, int *copy_back);
int   rkb_stage_out_finish(rkb_handle *h, void *user, const void *dev, size_t bytes, int copy_back);

/* Wait for the handle's stream with the ROCKET_WAIT_MS deadline (default 8 s),
 * then check the CUDA error state and the kernel error word.  Returns 0 or
 * ROCKET_E_DEVICE (with a log line naming `who`). */
int rkb_finish(rkb_handle *h, const char *who);

/* Profiler brackets: begin returns a slot (or -1 when profiling is off);
 * end records the closing event for kernel family `fam`. */
int  rkb_prof_begin(rkb_handle *h);
void rkb_prof_end(rkb_handle *h, int slot, int fam);

/* Deferred completion requested by this host thread (rocket_b200_set_async). */
int  rkb_async_enabled(void);

/* Count one device-reaching call and the kernels it launched. */
void rkb_count(uint64_t calls, uint64_t kernels);

/* ---- compute helpers shared by one-shot, resident and multi-GPU paths ----
 * All enqueue on h->stream and do not wait; the caller ends with rkb_finish. */

/* Dense GEMM on device operands. */
int rkb_dense_on(rkb_handle *h, int in_kind, int out_kind, int M, int N, int K,
                 const void *dA, long lda, const void *dB, long ldb, void *dC, long ldc);

/* Group-wise GEMM on packed device codes dWq (rkb_wpack_codes layout, w_bits
 * 8 or 4).  dA is int8 [M,K] on the device; a_scale [M*nG] and b_scale
 * [N*nG] may be host or device pointers (b_scale already offset to this
 * slice).  a_rows_const != 0 means a_scale[m*nG+g] does not depend on g, so A
 * stays exact in fp16 and the scale is applied per row in the epilogue. */
int rkb_gw_on(rkb_handle *h, int M, int N, int K, int group, int w_bits,
              const int8_t *dA, const float *a_scale, int a_rows_const,
              const void *dWq, const float *b_scale, void *dC, long ldc, int out_kind);

/* One dense GEMM call on operands anywhere (staged as needed).  finish = 0
 * leaves the call queued on the handle's stream for a later rkb_finish. */
int rkb_oneshot_dense(const char *who, int fd, int in_kind, int out_kind, int M, int K, int N,
                      const void *A, const void *B, void *C, int finish);

/* 1 if a host-resident a_scale [M*nG] is constant along g for every row. */
int rkb_rows_const(const float *a_scale, int M, int nG);

/* ---- composite-call plumbing (rkb_call.c) ---- */
#define RKB_CALL_MAX_TMP 64
typedef struct {
    rkb_handle *h;
    const char *who;
    void *tmp[RKB_CALL_MAX_TMP];
    int host_in;               /* an input was staged from host memory */
    int ntmp;
    int rc;
    struct { void *user; const void *dev; size_t bytes; } outs[4];
    int nouts;
} rkb_call;
int         rkb_call_begin(rkb_call *c, int fd, const char *who);
void       *rkb_call_tmp(rkb_call *c, size_t bytes);                      /* stream-ordered temporary */
const void *rkb_call_in(rkb_call *c, const void *user, size_t bytes);    /* device view of an input */
void       *rkb_call_out(rkb_call *c, void *user, size_t bytes);         /* device buffer for an output */
void        rkb_call_check(rkb_call *c, int rc);
int         rkb_call_end(rkb_call *c);                                   /* copy back, free, bounded wait */
/* fp16-input GEMM with fused epilogue: C = act(A W^T + bias) + residual (fp16 out) */
void        rkb_call_gemm(rkb_call *c, int M, int N, int K, const void *A, long lda, const void *W,
                          void *C, long ldc, const void *bias, int act, const void *res, long ldr);
/* any-kind GEMM on device operands with the call's temporaries for workspace */
void        rkb_call_gemm_kind(rkb_call *c, int in_kind, int out_kind, int M, int N, int K,
                               const void *A, long lda, const void *B, long ldb, void *C, long ldc);

/* Environment helpers (read on each call; cheap). */
long rkb_env_long(const char *name, long dflt);

#endif /* RKB_INTERNAL_H */
