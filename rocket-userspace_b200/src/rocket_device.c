/*
 * rocket_device.c -- the device shim: CUDA device handles in place of the
 * reference's /dev/accel fds (src/rocket_npu.c:470-892).
 *
 * A handle is a slot in a process-wide table: one CUDA device, one
 * non-blocking stream, a mapped pinned error word the kernels write when a
 * bounded wait expires, grow-only scratch buffers for staging host operands,
 * and a small BO table.  rocket_open() binds to ROCKET_DEV (default 0); the
 * multi-GPU paths open handles on explicit devices through rkb_open_on().
 */
#define _GNU_SOURCE
#include <errno.h>
#include <sched.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "rocket_b200.h"
#include "rkb_internal.h"

static rkb_handle g_h[RKB_MAX_HANDLES];
static pthread_mutex_t g_lock = PTHREAD_MUTEX_INITIALIZER;
static uint64_t g_calls, g_kernels;
static __thread int g_aff_base;
static long g_busy_poll_us = -1;

/* ---- profiler ------------------------------------------------------------ */
static int g_prof = -1;
static pthread_mutex_t g_prof_lock = PTHREAD_MUTEX_INITIALIZER;
static uint64_t g_prof_n[RKB_NKFAM];
static double g_prof_ms[RKB_NKFAM];
static const char *g_prof_name[RKB_NKFAM] = {
    "gemm_i8_tcgen05", "gemm_f16_tcgen05", "wgemm_w4_f16_tcgen05", "wgemm_w8_f16_tcgen05",
    "wgemm_w4_i8_tcgen05", "weight_pack", "act_prescale", "norm", "softmax", "attention",
    "elementwise", "wgemm_gw_i8_tcgen05"};

static int prof_on(void)
{
    if (g_prof < 0) g_prof = rkb_env_long("ROCKET_MM_PROFILE", 0) ? 1 : 0;
    return g_prof;
}

void rocket_b200_profile_enable(int on) { g_prof = on ? 1 : 0; }

void rocket_b200_profile_reset(void)
{
    pthread_mutex_lock(&g_prof_lock);
    memset(g_prof_n, 0, sizeof g_prof_n);
    memset(g_prof_ms, 0, sizeof g_prof_ms);
    pthread_mutex_unlock(&g_prof_lock);
}

int rocket_b200_profile_get(int idx, const char **name, uint64_t *launches, double *total_ms)
{
    if (idx < 0 || idx >= RKB_NKFAM) return ROCKET_E_SHAPE;
    pthread_mutex_lock(&g_prof_lock);
    if (name) *name = g_prof_name[idx];
    if (launches) *launches = g_prof_n[idx];
    if (total_ms) *total_ms = g_prof_ms[idx];
    pthread_mutex_unlock(&g_prof_lock);
    return 0;
}

int rkb_prof_begin(rkb_handle *h)
{
    if (!prof_on() || h->ev_used >= RKB_PROF_SLOTS) return -1;
    int s = h->ev_used;
    if (s >= h->ev_made) {
        if (cudaEventCreate(&h->ev[s][0]) != cudaSuccess || cudaEventCreate(&h->ev[s][1]) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        h->ev_made = s + 1;
    }
    cudaEventRecord(h->ev[s][0], h->stream);
    h->ev_used = s + 1;
    return s;
}

void rkb_prof_end(rkb_handle *h, int slot, int fam)
{
    if (slot < 0) return;
    cudaEventRecord(h->ev[slot][1], h->stream);
    h->ev_fam[slot] = fam;
}

static void prof_drain(rkb_handle *h)
{
    if (!h->ev_used) return;
    pthread_mutex_lock(&g_prof_lock);
    for (int s = 0; s < h->ev_used; s++) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, h->ev[s][0], h->ev[s][1]) == cudaSuccess) {
            g_prof_n[h->ev_fam[s]] += 1;
            g_prof_ms[h->ev_fam[s]] += ms;
        } else {
            cudaGetLastError();
        }
    }
    pthread_mutex_unlock(&g_prof_lock);
    h->ev_used = 0;
}

static __thread int g_async;
void rocket_b200_set_async(int on) { g_async = on ? 1 : 0; }
int  rkb_async_enabled(void) { return g_async; }

int rocket_b200_sync(int fd)
{
    rkb_handle *h = rkb_get(fd);
    if (!h) return ROCKET_E_DEVICE;
    return rkb_finish(h, "rocket_b200_sync");
}

void *rocket_b200_stream(int fd)
{
    rkb_handle *h = rkb_get(fd);
    return h ? (void *)h->stream : NULL;
}

int rocket_b200_device(int fd)
{
    rkb_handle *h = rkb_get(fd);
    return h ? h->device : ROCKET_E_DEVICE;
}

long rkb_env_long(const char *name, long dflt)
{
    const char *e = getenv(name);
    if (!e || !*e) return dflt;
    char *end;
    long v = strtol(e, &end, 10);
    return end == e ? dflt : v;
}

int rkb_device_count(void)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int rkb_open_on(int device)
{
    int ndev = rkb_device_count();
    if (ndev <= 0) return ROCKET_E_DEVICE;
    if (device < 0 || device >= ndev) return ROCKET_E_SHAPE;

    pthread_mutex_lock(&g_lock);
    int fd = -1;
    for (int i = 0; i < RKB_MAX_HANDLES; i++)
        if (!g_h[i].in_use) { fd = i; g_h[i].in_use = 1; break; }
    pthread_mutex_unlock(&g_lock);
    if (fd < 0) return ROCKET_E_NOMEM;

    rkb_handle *h = &g_h[fd];
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) goto fail;
    h->device = device;
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) goto fail;
    if (cudaHostAlloc((void **)&h->err_host, sizeof(int), cudaHostAllocMapped) != cudaSuccess) {
        cudaStreamDestroy(h->stream);
        goto fail;
    }
    *h->err_host = 0;
    cudaHostGetDevicePointer((void **)&h->err_dev, h->err_host, 0);
    cudaSetDevice(prev);
    return fd;
fail:
    ROCKET_LOGE("rocket_open: CUDA device %d unusable: %s\n", device,
                cudaGetErrorString(cudaGetLastError()));
    cudaSetDevice(prev);
    pthread_mutex_lock(&g_lock);
    memset(h, 0, sizeof *h);
    pthread_mutex_unlock(&g_lock);
    return ROCKET_E_DEVICE;
}

int rocket_open(void)
{
    return rkb_open_on((int)rkb_env_long("ROCKET_DEV", 0));
}

rkb_handle *rkb_get(int fd)
{
    if (fd < 0 || fd >= RKB_MAX_HANDLES || !g_h[fd].in_use) return NULL;
    rkb_handle *h = &g_h[fd];
    cudaSetDevice(h->device);
    return h;
}

void rocket_close(int fd)
{
    rkb_handle *h = rkb_get(fd);
    if (!h) return;
    cudaStreamSynchronize(h->stream);
    for (int i = 0; i < RKB_NSCR; i++) cudaFree(h->scr[i]);
    for (int i = 0; i <= RKB_NSCR; i++) {
        if (h->pin[i]) cudaFreeHost(h->pin[i]);
        if (h->pin_ev[i]) cudaEventDestroy(h->pin_ev[i]);
    }
    for (int i = 0; i < RKB_MAX_BOS; i++)
        if (h->bo[i].live) { cudaFree(h->bo[i].dptr); cudaFreeHost(h->bo[i].hptr); }
    for (int i = 0; i < h->ev_made; i++) {
        cudaEventDestroy(h->ev[i][0]);
        cudaEventDestroy(h->ev[i][1]);
    }
    cudaStreamDestroy(h->stream);
    cudaFreeHost(h->err_host);
    pthread_mutex_lock(&g_lock);
    memset(h, 0, sizeof *h);
    pthread_mutex_unlock(&g_lock);
}

void *rkb_scratch(rkb_handle *h, int slot, size_t bytes)
{
    if (bytes == 0) bytes = 16;
    if (h->scr_cap[slot] >= bytes) return h->scr[slot];
    /* the old buffer may still be read by queued work */
    cudaStreamSynchronize(h->stream);
    cudaFree(h->scr[slot]);
    h->scr[slot] = NULL;
    h->scr_cap[slot] = 0;
    size_t cap = (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;   /* 1 MiB granules */
    if (cudaMalloc(&h->scr[slot], cap) != cudaSuccess) {
        cudaGetLastError();
        ROCKET_LOGE("rkb: device scratch of %zu bytes failed\n", cap);
        return NULL;
    }
    h->scr_cap[slot] = cap;
    return h->scr[slot];
}

/* CUDA device owning p; -1 for pinned (or otherwise CUDA-known) host memory,
 * -2 for pageable host memory. */
static int ptr_kind(const void *p)
{
    struct cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return -2;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return a.device;
    return a.type == cudaMemoryTypeUnregistered ? -2 : -1;
}

int rkb_ptr_device(const void *p)
{
    const int k = ptr_kind(p);
    return k >= 0 ? k : -1;
}

/* Pageable operands up to this size go through a pinned bounce buffer: one
 * host memcpy plus an asynchronous DMA instead of the driver's synchronous
 * staging of pageable memory.  Larger ones are copied directly. */
#define RKB_BOUNCE_MAX ((size_t)8 << 20)

/* Pinned buffer `slot` of at least `bytes`, free of queued copies. */
static void *pin_slot(rkb_handle *h, int slot, size_t bytes)
{
    if (h->pin_ev[slot]) cudaEventSynchronize(h->pin_ev[slot]);
    if (h->pin_cap[slot] < bytes) {
        if (h->pin[slot]) cudaFreeHost(h->pin[slot]);
        h->pin[slot] = NULL;
        h->pin_cap[slot] = 0;
        size_t cap = (bytes + 0xFFFF) & ~(size_t)0xFFFF;
        if (cudaHostAlloc(&h->pin[slot], cap, cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            return NULL;
        }
        h->pin_cap[slot] = cap;
    }
    if (!h->pin_ev[slot] &&
        cudaEventCreateWithFlags(&h->pin_ev[slot], cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        h->pin_ev[slot] = NULL;
        return NULL;
    }
    return h->pin[slot];
}

const void *rkb_stage_in(rkb_handle *h, int slot, const void *user, size_t bytes)
{
    const int kind = ptr_kind(user);
    if (kind == h->device && ((uintptr_t)user & 15) == 0) return user;
    void *d = rkb_scratch(h, slot, bytes);
    if (!d) return NULL;
    const void *src = user;
    void *p = (kind == -2 && bytes <= RKB_BOUNCE_MAX) ? pin_slot(h, slot, bytes) : NULL;
    if (p) {
        memcpy(p, user, bytes);
        src = p;
    }
    if (cudaMemcpyAsync(d, src, bytes, cudaMemcpyDefault, h->stream) != cudaSuccess) {
        ROCKET_LOGE("rkb: input copy failed: %s\n", cudaGetErrorString(cudaGetLastError()));
        return NULL;
    }
    if (p) cudaEventRecord(h->pin_ev[slot], h->stream);
    return d;
}

void *rkb_stage_out(rkb_handle *h, int slot, void *user, size_t bytes, int *copy_back)
{
    if (rkb_ptr_device(user) == h->device && ((uintptr_t)user & 15) == 0) {
        *copy_back = 0;
        return user;
    }
    *copy_back = 1;
    return rkb_scratch(h, slot, bytes);
}

int rkb_stage_out_finish(rkb_handle *h, void *user, const void *dev, size_t bytes, int copy_back)
{
    if (!copy_back) return 0;
    /* a small pageable output lands in the pinned bounce buffer and is copied
     * out by rkb_finish once the stream is done (one output per wait) */
    if (h->npend == 0 && bytes <= RKB_BOUNCE_MAX && ptr_kind(user) == -2) {
        void *p = pin_slot(h, RKB_NSCR, bytes);
        if (p && cudaMemcpyAsync(p, dev, bytes, cudaMemcpyDeviceToHost, h->stream) == cudaSuccess) {
            cudaEventRecord(h->pin_ev[RKB_NSCR], h->stream);
            h->pend.user = user;
            h->pend.pin = p;
            h->pend.bytes = bytes;
            h->npend = 1;
            return 0;
        }
        cudaGetLastError();
    }
    if (cudaMemcpyAsync(user, dev, bytes, cudaMemcpyDefault, h->stream) != cudaSuccess) {
        ROCKET_LOGE("rkb: output copy failed: %s\n", cudaGetErrorString(cudaGetLastError()));
        return ROCKET_E_DEVICE;
    }
    return 0;
}

static uint64_t now_ns(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

/* Completion wait: spin on cudaStreamQuery for the busy-poll window
 * (ROCKET_BUSY_POLL us, default 20000), then poll every 50 us, giving up at the
 * ROCKET_WAIT_MS deadline (default 8000) -- the analogue of the reference's
 * fence wait (src/rocket_matmul.c:53-69, src/rocket_npu.c:682-725). */
static int wait_stream(rkb_handle *h, uint64_t timeout_ns)
{
    const uint64_t t0 = now_ns();
    long bp = g_busy_poll_us >= 0 ? g_busy_poll_us : rkb_env_long("ROCKET_BUSY_POLL", 20000);
    for (;;) {
        cudaError_t e = cudaStreamQuery(h->stream);
        if (e == cudaSuccess) return 0;
        if (e != cudaErrorNotReady) return ROCKET_E_DEVICE;
        uint64_t dt = now_ns() - t0;
        if (dt > timeout_ns) return -EBUSY;
        if (dt > (uint64_t)bp * 1000ull) usleep(50);
        else sched_yield();
    }
}

int rkb_finish(rkb_handle *h, const char *who)
{
    uint64_t to = (uint64_t)rkb_env_long("ROCKET_WAIT_MS", 8000) * 1000000ull;
    int rc = wait_stream(h, to);
    const int npend = h->npend;
    h->npend = 0;
    if (rc == 0 && npend) memcpy(h->pend.user, h->pend.pin, h->pend.bytes);
    if (rc == -EBUSY) {
        ROCKET_LOGE("%s: WAIT TIMEOUT after %llu ms\n", who, (unsigned long long)(to / 1000000ull));
        return ROCKET_E_DEVICE;
    }
    cudaError_t e = cudaGetLastError();
    if (rc || e != cudaSuccess) {
        ROCKET_LOGE("%s: CUDA error: %s\n", who, cudaGetErrorString(e != cudaSuccess ? e : cudaStreamQuery(h->stream)));
        return ROCKET_E_DEVICE;
    }
    prof_drain(h);
    int ew = *(volatile int *)h->err_host;
    if (ew) {
        ROCKET_LOGE("%s: kernel pipeline wait expired (code %d)\n", who, ew);
        *(volatile int *)h->err_host = 0;
        return ROCKET_E_DEVICE;
    }
    return 0;
}

void rkb_count(uint64_t calls, uint64_t kernels)
{
    __atomic_add_fetch(&g_calls, calls, __ATOMIC_RELAXED);
    __atomic_add_fetch(&g_kernels, kernels, __ATOMIC_RELAXED);
}

uint64_t rocket_submit_ioctl_count(void) { return __atomic_load_n(&g_calls, __ATOMIC_RELAXED); }
uint64_t rocket_submit_task_count(void) { return __atomic_load_n(&g_kernels, __ATOMIC_RELAXED); }
void rocket_submit_counters_reset(void)
{
    __atomic_store_n(&g_calls, 0, __ATOMIC_RELAXED);
    __atomic_store_n(&g_kernels, 0, __ATOMIC_RELAXED);
}

/* ---- affinity: stored, never applied (no big.LITTLE host) ---------------- */
void rocket_affinity_set_base(int base) { g_aff_base = base; }
int  rocket_affinity_get_base(void) { return g_aff_base; }
void rocket_pin_worker(int worker_idx) { (void)worker_idx; }
int  rocket_num_big_cores(void) { return 0; }

/* ---- buffer objects ----------------------------------------------------- */
int rocket_bo_alloc(int fd, size_t size, rocket_bo *bo)
{
    rkb_handle *h = rkb_get(fd);
    if (!h || !bo || size == 0) return -EINVAL;
    int slot = -1;
    for (int i = 0; i < RKB_MAX_BOS; i++)
        if (!h->bo[i].live) { slot = i; break; }
    if (slot < 0) return -ENOMEM;
    size = (size + 4095) & ~(size_t)4095;
    void *d = NULL, *p = NULL;
    if (cudaMalloc(&d, size) != cudaSuccess) { cudaGetLastError(); return -ENOMEM; }
    if (cudaHostAlloc(&p, size, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(d);
        return -ENOMEM;
    }
    memset(p, 0, size);
    cudaMemset(d, 0, size);
    h->bo[slot].dptr = d;
    h->bo[slot].hptr = p;
    h->bo[slot].size = size;
    h->bo[slot].live = 1;
    bo->handle = (uint32_t)slot;
    bo->dma_address = (uint64_t)(uintptr_t)d;
    bo->mmap_offset = 0;
    bo->size = size;
    bo->ptr = p;
    return 0;
}

void rocket_bo_free(int fd, rocket_bo *bo)
{
    rkb_handle *h = rkb_get(fd);
    if (!h || !bo || bo->handle >= RKB_MAX_BOS || !h->bo[bo->handle].live) return;
    cudaStreamSynchronize(h->stream);
    cudaFree(h->bo[bo->handle].dptr);
    cudaFreeHost(h->bo[bo->handle].hptr);
    memset(&h->bo[bo->handle], 0, sizeof h->bo[0]);
    memset(bo, 0, sizeof *bo);
}

static int bo_check(rkb_handle *h, const rocket_bo *bo)
{
    return h && bo && bo->handle < RKB_MAX_BOS && h->bo[bo->handle].live &&
           h->bo[bo->handle].hptr == bo->ptr;
}

static int ranges_ok(const rocket_bo *bo, const rocket_bo_range *r, unsigned n)
{
    uint64_t end = 0;
    for (unsigned i = 0; i < n; i++) {
        if (r[i].size == 0 || r[i].offset < end || r[i].offset + r[i].size > bo->size) return 0;
        end = r[i].offset + r[i].size;
    }
    return 1;
}

int rocket_bo_prep_ranges(int fd, rocket_bo *bo, const rocket_bo_range *r, unsigned n,
                          uint64_t timeout_ns)
{
    rkb_handle *h = rkb_get(fd);
    if (!bo_check(h, bo)) return -EINVAL;
    if (n && !ranges_ok(bo, r, n)) return -EINVAL;
    int rc = wait_stream(h, timeout_ns);
    if (rc) return rc == -EBUSY ? -EBUSY : -EIO;
    const uint8_t *d = h->bo[bo->handle].dptr;
    uint8_t *p = bo->ptr;
    if (n == 0) {
        if (cudaMemcpy(p, d, bo->size, cudaMemcpyDeviceToHost) != cudaSuccess) return -EIO;
    } else {
        for (unsigned i = 0; i < n; i++)
            if (cudaMemcpy(p + r[i].offset, d + r[i].offset, r[i].size, cudaMemcpyDeviceToHost) != cudaSuccess)
                return -EIO;
    }
    return 0;
}

int rocket_bo_prep(int fd, rocket_bo *bo, int dir, uint64_t timeout_ns)
{
    if (dir == 1) {
        rkb_handle *h = rkb_get(fd);
        return bo_check(h, bo) ? 0 : -EINVAL;
    }
    return rocket_bo_prep_ranges(fd, bo, NULL, 0, timeout_ns);
}

int rocket_bo_fini_ranges(int fd, rocket_bo *bo, const rocket_bo_range *r, unsigned n)
{
    rkb_handle *h = rkb_get(fd);
    if (!bo_check(h, bo)) return -EINVAL;
    if (n && !ranges_ok(bo, r, n)) return -EINVAL;
    uint8_t *d = h->bo[bo->handle].dptr;
    const uint8_t *p = bo->ptr;
    if (n == 0) {
        if (cudaMemcpyAsync(d, p, bo->size, cudaMemcpyHostToDevice, h->stream) != cudaSuccess) return -EIO;
    } else {
        for (unsigned i = 0; i < n; i++)
            if (cudaMemcpyAsync(d + r[i].offset, p + r[i].offset, r[i].size, cudaMemcpyHostToDevice,
                                h->stream) != cudaSuccess)
                return -EIO;
    }
    return 0;
}

int rocket_bo_fini(int fd, rocket_bo *bo) { return rocket_bo_fini_ranges(fd, bo, NULL, 0); }

int  rocket_bo_ranges_supported(void) { return 1; }
int  rocket_batched_submit_supported(void) { return 0; }
int  rocket_ppu_done_supported(void) { return 0; }
int  rocket_batch_completion_tracked(void) { return 0; }
void rocket_busy_poll_set_us(long us) { g_busy_poll_us = us < 0 ? 0 : us; }

/* ---- register-program submission: not a GPU concept --------------------- */
int rocket_submit_matmul(int fd, const rocket_bo *rb, uint32_t c, const uint32_t *i, uint32_t ni,
                         const uint32_t *o, uint32_t no, uint32_t t)
{
    (void)fd; (void)rb; (void)c; (void)i; (void)ni; (void)o; (void)no; (void)t;
    return ROCKET_E_UNSUPPORTED;
}
int rocket_submit_matmul_flags(int fd, const rocket_bo *rb, uint32_t c, const uint32_t *i,
                               uint32_t ni, const uint32_t *o, uint32_t no, uint32_t f)
{
    (void)fd; (void)rb; (void)c; (void)i; (void)ni; (void)o; (void)no; (void)f;
    return ROCKET_E_UNSUPPORTED;
}
int rocket_submit_tasks(int fd, const rocket_task_desc *t, uint32_t n, const uint32_t *i,
                        uint32_t ni, const uint32_t *o, uint32_t no)
{
    (void)fd; (void)t; (void)n; (void)i; (void)ni; (void)o; (void)no;
    return ROCKET_E_UNSUPPORTED;
}
int rocket_submit_tasks_flags(int fd, const rocket_task_desc *t, uint32_t n, const uint32_t *i,
                              uint32_t ni, const uint32_t *o, uint32_t no, uint32_t f)
{
    (void)fd; (void)t; (void)n; (void)i; (void)ni; (void)o; (void)no; (void)f;
    return ROCKET_E_UNSUPPORTED;
}
size_t rocket_submit_scratch_size(uint32_t max_tasks) { return (size_t)max_tasks * 16; }
int rocket_submit_tasks_pre(int fd, void *s, const rocket_task_desc *t, uint32_t n,
                            const uint32_t *i, uint32_t ni, const uint32_t *o, uint32_t no,
                            uint32_t f)
{
    (void)fd; (void)s; (void)t; (void)n; (void)i; (void)ni; (void)o; (void)no; (void)f;
    return ROCKET_E_UNSUPPORTED;
}
int rocket_submit_jobs(int fd, const rocket_job_desc *j, uint32_t n)
{
    (void)fd; (void)j; (void)n;
    return ROCKET_E_UNSUPPORTED;
}
