/*
 * rocket_hw_profile.h -- the hardware-profile query of librocketnpu, B200
 * build (reference include/rocket_hw_profile.h:60-108).  The reference selects
 * an NPU profile (CBUF geometry, tile cap, dtype mask) from the device tree;
 * its callers read max_tile to reason about resident-weight tiling.  Here
 * there is one profile, "b200", describing the tiles the B200 kernels use.
 * The struct layout is the reference's, so callers compiled against either
 * header read the same fields.
 */
#ifndef ROCKET_HW_PROFILE_H
#define ROCKET_HW_PROFILE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct rocket_hw_profile {
    const char *name;          /* "b200" */
    int cbuf_banks;            /* NPU conv-buffer banks: 0 (no such buffer) */
    int cbuf_bank_size;        /* 0 */
    int max_tile;              /* widest output tile edge of the GEMM kernels (256) */
    int kgroup_2b;             /* K step of one MMA for 2-byte operands (16) */
    int kgroup_4b;             /* K step of one MMA for 4-byte (tf32) operands (8) */
    int ngroup;                /* N granularity of an MMA (16) */
    uint32_t dtype_supported;  /* all precisions the library serves: ~0u */
    const char *select_warning;/* NULL */
    int default_workers;       /* default worker count of a resident context (1) */
};

/* The active profile (always the "b200" one). */
const struct rocket_hw_profile *rocket_hw_current(void);
/* The profile named `name`, or NULL ("b200" is the only one). */
const struct rocket_hw_profile *rocket_hw_by_name(const char *name);

#ifdef __cplusplus
}
#endif
#endif
