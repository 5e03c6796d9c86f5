/*
 * rocket_npu.h -- device shim of the B200 build of librocketnpu.
 *
 * The reference library opens /dev/accel/accel0 (the RK3588 "rocket" DRM-accel
 * driver) and moves register-command programs through CREATE_BO / SUBMIT /
 * PREP_BO / FINI_BO ioctls.  This build keeps the same C entry points so a
 * caller links unchanged, and maps each one onto CUDA:
 *
 *   rocket_open()          -> a small non-negative handle bound to one CUDA
 *                             device (ROCKET_DEV, default 0) with its own
 *                             non-blocking stream, device scratch pool and a
 *                             device error word for bounded in-kernel waits.
 *   rocket_bo_alloc()      -> device memory (dma_address = device pointer) plus
 *                             a pinned host mirror (ptr).
 *   rocket_bo_fini()       -> host mirror -> device copy   ("flush for device").
 *   rocket_bo_prep(dir=0)  -> stream sync + device -> host  ("invalidate").
 *   rocket_submit_*()      -> ROCKET_E_UNSUPPORTED: there are no NPU register
 *                             programs on a GPU; the matmul entry points in
 *                             rocket_matmul.h launch sm_100a kernels instead.
 *
 * Reference interface: include/rocket_npu.h (status enum :41-48, rocket_bo
 * :51-57, open/close :65-66, BO API :107-119, submit API :150-293, counters
 * :295-304) and src/rocket_npu.c:470-892.
 */
#ifndef ROCKET_NPU_H
#define ROCKET_NPU_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status vocabulary shared by every int-returning entry point (reference
 * include/rocket_npu.h:41-48).  `ret < 0` is the one failure test; the matmul
 * *_plan() previews return a positive tile count on success. */
enum rocket_status {
    ROCKET_OK            =  0,
    ROCKET_E_SHAPE       = -1,
    ROCKET_E_TILING      = -2,  /* also "weight must be re-packed" on resident paths */
    ROCKET_E_NOMEM       = -3,
    ROCKET_E_DEVICE      = -4,  /* CUDA error, or a bounded in-kernel wait expired */
    ROCKET_E_UNSUPPORTED = -5,
};

/* A buffer object (reference include/rocket_npu.h:51-57).  On B200:
 *   handle      -- slot index inside the owning device handle
 *   dma_address -- the device pointer (cast to uint64_t)
 *   ptr         -- pinned host mirror, valid after rocket_bo_alloc */
typedef struct {
    uint32_t handle;
    uint64_t dma_address;
    uint64_t mmap_offset;
    size_t   size;
    void    *ptr;
} rocket_bo;

/* Open a device handle.  Returns a handle >= 0, or a negative rocket_status
 * (ROCKET_E_DEVICE when no CUDA device is visible).  Replaces
 * src/rocket_npu.c:470-525. */
int  rocket_open(void);
void rocket_close(int fd);

/* CPU-affinity hints (reference include/rocket_npu.h:84-98).  The B200 build
 * has no big.LITTLE host to pin to: the base is stored and returned, pinning
 * is a no-op and rocket_num_big_cores() returns 0 ("pinning disabled"). */
void rocket_affinity_set_base(int base);
int  rocket_affinity_get_base(void);
void rocket_pin_worker(int worker_idx);
int  rocket_num_big_cores(void);

/* Buffer objects (reference include/rocket_npu.h:107-119, src/rocket_npu.c:538-739). */
int  rocket_bo_alloc(int fd, size_t size, rocket_bo *bo);
void rocket_bo_free(int fd, rocket_bo *bo);
/* dir 0: wait for the handle's stream (bounded by timeout_ns; 0 = poll, returns
 * -EBUSY while work is pending) then copy device -> host mirror.
 * dir 1: nothing to do before a CPU write (rocket_bo_fini publishes it). */
int  rocket_bo_prep(int fd, rocket_bo *bo, int dir, uint64_t timeout_ns);
/* Copy the host mirror to the device (the "flush for the device" step). */
int  rocket_bo_fini(int fd, rocket_bo *bo);

typedef struct { uint64_t offset, size; } rocket_bo_range;
/* Ranged forms: ranges ascending, non-overlapping, inside the BO, else -EINVAL
 * (reference include/rocket_npu.h:132-135).  n == 0 means the whole object. */
int  rocket_bo_prep_ranges(int fd, rocket_bo *bo, const rocket_bo_range *r,
                           unsigned n, uint64_t timeout_ns);
int  rocket_bo_fini_ranges(int fd, rocket_bo *bo, const rocket_bo_range *r,
                           unsigned n);

/* Capability probes (reference include/rocket_npu.h:139-167).  Ranged cache
 * maintenance is supported (1); NPU job chaining / PPU completion / batched
 * completion tracking do not exist on a GPU (0). */
int  rocket_bo_ranges_supported(void);
int  rocket_batched_submit_supported(void);
int  rocket_ppu_done_supported(void);
int  rocket_batch_completion_tracked(void);
void rocket_busy_poll_set_us(long us);

/* Register-program submission (reference include/rocket_npu.h:180-293).
 * Every form returns ROCKET_E_UNSUPPORTED: a GPU runs kernels, not NPU
 * register-command programs. */
#define ROCKET_JOB_BATCHED      (1u << 0)
#define ROCKET_JOB_NO_DPU_DONE  (1u << 1)
#define ROCKET_JOB_PPU_DONE     (1u << 2)

typedef struct { uint32_t regcmd; uint32_t regcmd_count; } rocket_task_desc;
typedef struct {
    const rocket_task_desc *tasks;  uint32_t n_tasks;
    const uint32_t *in_handles;     uint32_t n_in;
    const uint32_t *out_handles;    uint32_t n_out;
} rocket_job_desc;

int  rocket_submit_matmul(int fd, const rocket_bo *regcmd_bo, uint32_t regcmd_count,
                          const uint32_t *in_handles, uint32_t n_in,
                          const uint32_t *out_handles, uint32_t n_out,
                          uint32_t timeout_ms);
int  rocket_submit_matmul_flags(int fd, const rocket_bo *regcmd_bo, uint32_t regcmd_count,
                                const uint32_t *in_handles, uint32_t n_in,
                                const uint32_t *out_handles, uint32_t n_out,
                                uint32_t job_flags);
int  rocket_submit_tasks(int fd, const rocket_task_desc *tasks, uint32_t n_tasks,
                         const uint32_t *in_handles, uint32_t n_in,
                         const uint32_t *out_handles, uint32_t n_out);
int  rocket_submit_tasks_flags(int fd, const rocket_task_desc *tasks, uint32_t n_tasks,
                               const uint32_t *in_handles, uint32_t n_in,
                               const uint32_t *out_handles, uint32_t n_out,
                               uint32_t job_flags);
size_t rocket_submit_scratch_size(uint32_t max_tasks);
int  rocket_submit_tasks_pre(int fd, void *scratch,
                             const rocket_task_desc *tasks, uint32_t n_tasks,
                             const uint32_t *in_handles, uint32_t n_in,
                             const uint32_t *out_handles, uint32_t n_out,
                             uint32_t job_flags);
int  rocket_submit_jobs(int fd, const rocket_job_desc *jobs, uint32_t n_jobs);

/* Process-wide launch counters (reference include/rocket_npu.h:295-304).  On
 * B200 "ioctl" counts library entry calls that reached the device and "task"
 * counts kernels launched by them, so a caller can see how many launches a
 * call cost. */
uint64_t rocket_submit_ioctl_count(void);
uint64_t rocket_submit_task_count(void);
void     rocket_submit_counters_reset(void);

#ifdef __cplusplus
}
#endif
#endif /* ROCKET_NPU_H */
