"""N-column sharding across ranks -- the multi-GPU form of the reference's
worker split (src/rocket_prepacked_int8.c:161-165: each worker computes
C[:, n0:n0+nsub] from the full A, slices rounded up to the dtype's N atom).

One process per GPU: rank r holds weight rows [n0, n0+nsub) and the full A,
computes its column slice with no collective, and -- only when a caller needs
the full output on every rank -- the slices are all-gathered (NCCL over
NVLink on GPUs, gloo on CPU) and interleaved back into row-major [M, N].
"""
from __future__ import annotations


def shard(n: int, world: int, rank: int, atom: int = 32) -> tuple[int, int]:
    """(n0, nsub) of rank's column slice: ceil(n / world) rounded up to `atom`."""
    step = -(-n // world)
    step = -(-step // atom) * atom
    n0 = rank * step
    return n0, max(0, min(step, n - n0))


def max_slice(n: int, world: int, atom: int = 32) -> int:
    return shard(n, world, 0, atom)[1]


def gather_columns(local, n: int, world: int, group=None, atom: int = 32):
    """All-gather every rank's [M, nsub] slice and return the full [M, n]
    output (torch tensors; works for any torch.distributed backend)."""
    import torch
    import torch.distributed as dist
    m = local.shape[0]
    w = max_slice(n, world, atom)
    padded = torch.zeros((m, w), dtype=local.dtype, device=local.device)
    padded[:, :local.shape[1]] = local
    parts = torch.empty((world, m, w), dtype=local.dtype, device=local.device)
    if local.device.type == "cuda":
        dist.all_gather_into_tensor(parts, padded, group=group)   # NCCL over NVLink
    else:
        dist.all_gather(list(parts.unbind(0)), padded, group=group)
    out = torch.empty((m, n), dtype=local.dtype, device=local.device)
    for r in range(world):
        n0, ns = shard(n, world, r, atom)
        if ns:
            out[:, n0:n0 + ns] = parts[r, :, :ns]
    return out
