// rkb_wlayout.cuh -- addressing of the resident quantised-weight layout.
//
// Codes (and, for the fast group-wise form, fp16 scales) are stored in 256-row
// N tiles.  Inside tile t, each 64-wide K block is one contiguous block of
// rows_t rows (row-major): 64 codes per row (int8: 64 bytes, int4: 32 bytes)
// or 2 fp16 scales per row (4 bytes).  Every tile but the last holds 256
// rows; the last holds only the remaining rows, rounded up to 32, so a
// weight's footprint is its own rows (plus K padded to 128), not a multiple
// of 256 rows.  K is padded to a multiple of 128 (nkb = that / 64 blocks).
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace rkb {

constexpr int WL_TILE = 256;

// rows stored in tile t of an N-row weight
__host__ __device__ inline int wl_rows(int N, int t) {
    int r = N - t * WL_TILE;
    r = r > WL_TILE ? WL_TILE : r;
    return (r + 31) & ~31;
}
__host__ __device__ inline int wl_nkb(int K) { return (K + 127) / 128 * 2; }
__host__ __device__ inline int wl_ntiles(int N) { return (N + WL_TILE - 1) / WL_TILE; }
// byte offset of block (t, kb) for rows of row_bytes bytes
__host__ __device__ inline size_t wl_block(int N, int nkb, int t, int kb, int row_bytes) {
    return (static_cast<size_t>(t) * nkb * WL_TILE + static_cast<size_t>(kb) * wl_rows(N, t)) * row_bytes;
}
// total bytes
__host__ __device__ inline size_t wl_bytes(int N, int K, int row_bytes) {
    const int nt = wl_ntiles(N);
    if (nt == 0) return 0;
    return (static_cast<size_t>(nt - 1) * WL_TILE + wl_rows(N, nt - 1)) * wl_nkb(K) * row_bytes;
}

}  // namespace rkb
