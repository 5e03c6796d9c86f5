"""CPU, world size 2 over gloo: the N-column sharding and the output gather
that bench.py --gpus N uses reproduce the unsharded result exactly."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, K, N, q):
    import sys
    import torch
    import torch.distributed as dist
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    import importlib.util
    spec = importlib.util.spec_from_file_location("shard", os.path.join(repo, "rocket-userspace_b200", "shard.py"))
    shard = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(shard)
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    A = oracle.uniform_i8(1, -128, 127, (M, K))
    B = oracle.uniform_i8(2, -128, 127, (N, K))
    n0, ns = shard.shard(N, world, rank)
    local = oracle.matmul_int8(A, np.ascontiguousarray(B[n0:n0 + ns])) if ns else np.zeros((M, 0), np.int32)
    full = shard.gather_columns(torch.from_numpy(local), N, world)
    if rank == 0:
        q.put(full.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("N", [256, 5888, 96])
def test_sharded_gather_equals_full(N):
    M, K, world = 16, 64, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, K, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    import oracle
    A = oracle.uniform_i8(1, -128, 127, (M, K))
    B = oracle.uniform_i8(2, -128, 127, (N, K))
    assert np.array_equal(full, oracle.matmul_int8(A, B))


def test_shard_rule_matches_reference_split():
    import importlib.util
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("shard", os.path.join(repo, "rocket-userspace_b200", "shard.py"))
    shard = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(shard)
    for N, world in [(5888, 8), (3840, 3), (30720, 8), (64, 4)]:
        parts = [shard.shard(N, world, r) for r in range(world)]
        assert sum(ns for _, ns in parts) == N
        assert all(n0 % 32 == 0 for n0, _ in parts)
        covered = sorted((n0, n0 + ns) for n0, ns in parts if ns)
        assert covered[0][0] == 0 and covered[-1][1] == N
        assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))
