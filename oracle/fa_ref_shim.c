/* TEST INFRASTRUCTURE ONLY: the reference's host reference for masked GQA
 * attention (rocket_flash_attn_ref_fp16, src/rocket_attn.c:189-222) provided by
 * the oracle's restatement, threaded over (head, token) rows.  The restatement
 * is pinned bit for bit against the reference's own function
 * (tests/test_oracle_fa.py); threading changes no result (rows are
 * independent).  Linked into the reference's flash-attention gate so its long
 * context cases check in seconds instead of many minutes. */
#include <stdint.h>
#include <unistd.h>

#include "oracle.h"

void rocket_flash_attn_ref_fp16(int n_tokens, int n_kv, int head_dim, int dv, int n_head, int n_kv_heads,
                                float scale, float softcap, const _Float16 *Q, const _Float16 *K,
                                const _Float16 *V, const _Float16 *mask, _Float16 *out)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    orc_flash_attn_f16_mt(n_tokens, n_kv, head_dim, dv, n_head, n_kv_heads, scale, softcap,
                          (const uint16_t *)Q, (const uint16_t *)K, (const uint16_t *)V,
                          (const uint16_t *)mask, (uint16_t *)out, n > 0 ? (int)n : 1);
}
