"""GPU: the allocation-free group-wise int4 entry point.

rocket_b200_matmul_int4_groupwise_noalloc serves callers that may not call
cudaMalloc (runtimes that own all device memory, fixed memory budgets, loops
that must not allocate): its scratch is a fixed array inside the library.  It
computes the fast group-wise form (w * b_scale rounded to fp16 before the
MMA), so it must agree with rocket_matmul_int4_groupwise and with the exact
definition within that form's bound (1e-2 Frobenius, 2e-2 max relative), call
after call (the array keeps the previous call's contents).
This file is collected last so a stop-at-first-failure run has already run
every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_FRO = 1e-2
MAX_ABS_REL = 2e-2


def test_noalloc_matches_existing_entry_twice(rkb, dev, orc):
    import torch
    fn = rkb.lib.rocket_b200_matmul_int4_groupwise_noalloc
    torch.cuda.set_device(0)
    for call, (M, K, N, group) in enumerate([(128, 1024, 512, 32), (64, 512, 256, 128)]):
        nG = K // group
        A = torch.from_numpy(orc.uniform_i8(300 + call, -127, 127, (M, K))).cuda()
        B = torch.from_numpy(orc.uniform_i8(400 + call, -8, 7, (N, K))).cuda()
        a = torch.from_numpy(orc.uniform_f32(500 + call, 0.5, 1.5, (M, nG))).cuda()
        b = torch.from_numpy(orc.uniform_f32(600 + call, 0.005, 0.02, (N, nG))).cuda()
        C_ref = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        assert dev.matmul_int4_groupwise(M, K, N, A, B, a, b, C_ref, group) == 0
        C = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        assert fn(M, K, N, rkb.ptr(A), rkb.ptr(B), rkb.ptr(a), rkb.ptr(b), rkb.ptr(C), group, None) == 0
        torch.cuda.synchronize()
        got, ref = C.cpu().numpy(), C_ref.cpu().numpy()
        assert np.isfinite(got).all()
        assert orc.rel_frobenius(got, ref) <= REL_FRO and orc.max_abs_rel(got, ref) <= MAX_ABS_REL
        exact = orc.gw_ref(A.cpu().numpy(), B.cpu().numpy(), a.cpu().numpy(), b.cpu().numpy(), group)
        assert orc.rel_frobenius(got, exact) <= REL_FRO and orc.max_abs_rel(got, exact) <= MAX_ABS_REL


def test_noalloc_rejects_oversize_and_host_memory(rkb, dev):
    import torch
    fn = rkb.lib.rocket_b200_matmul_int4_groupwise_noalloc
    M, K, N, group = 4096, 4096, 8192, 32   # needs ~48 MiB of scratch > 32 MiB
    A = torch.zeros((M, K), dtype=torch.int8, device="cuda")
    B = torch.zeros((N, K), dtype=torch.int8, device="cuda")
    a = torch.ones((M, K // group), device="cuda")
    b = torch.ones((N, K // group), device="cuda")
    C = torch.zeros((M, N), device="cuda")
    assert fn(M, K, N, rkb.ptr(A), rkb.ptr(B), rkb.ptr(a), rkb.ptr(b), rkb.ptr(C), group, None) == rkb.ROCKET_E_NOMEM
    h = np.zeros((64, 64), np.int8)
    hs = np.ones((64, 2), np.float32)
    hc = np.zeros((64, 64), np.float32)
    assert fn(64, 64, 64, rkb.ptr(h), rkb.ptr(h), rkb.ptr(hs), rkb.ptr(hs), rkb.ptr(hc), 32, None) == rkb.ROCKET_E_SHAPE
