/*
 * ref_npu_stub.c -- TEST INFRASTRUCTURE ONLY.  Stands in for the reference's
 * DRM shim (src/rocket_npu.c, which needs libdrm and the rocket accel uAPI
 * header) so the reference's other sources link into oracle/_ref/libref.so.
 * No device is ever present: rocket_open() fails with -ENODEV, which is all the
 * reference's host-reference functions (*_ref_fp16) need -- they never touch it.
 */
#include <errno.h>
#include <stddef.h>
#include <stdint.h>

int rocket_open(void) { return -ENODEV; }
void rocket_close(int fd) { (void)fd; }
int rocket_bo_alloc(int fd, size_t size, void *bo) { (void)fd; (void)size; (void)bo; return -ENODEV; }
void rocket_bo_free(int fd, void *bo) { (void)fd; (void)bo; }
int rocket_bo_prep(int fd, void *bo, int dir, uint64_t t) { (void)fd; (void)bo; (void)dir; (void)t; return -ENODEV; }
int rocket_bo_fini(int fd, void *bo) { (void)fd; (void)bo; return -ENODEV; }
int rocket_bo_prep_ranges(int fd, void *bo, const void *r, unsigned n, uint64_t t) { (void)fd; (void)bo; (void)r; (void)n; (void)t; return -ENODEV; }
int rocket_bo_fini_ranges(int fd, void *bo, const void *r, unsigned n) { (void)fd; (void)bo; (void)r; (void)n; return -ENODEV; }
int rocket_bo_ranges_supported(void) { return 0; }
int rocket_batched_submit_supported(void) { return 0; }
int rocket_ppu_done_supported(void) { return 0; }
int rocket_batch_completion_tracked(void) { return 0; }
int rocket_submit_matmul(void) { return -ENODEV; }
int rocket_submit_matmul_flags(void) { return -ENODEV; }
size_t rocket_submit_scratch_size(uint32_t n) { return (size_t)n * 64; }
int rocket_submit_tasks(void) { return -ENODEV; }
int rocket_submit_tasks_flags(void) { return -ENODEV; }
int rocket_submit_tasks_pre(void) { return -ENODEV; }
