"""GPU parity: the CUDA path through the C ABI against the oracle and the
golden fixtures made by the reference's own gates.

Tolerances (north-star): int8 / int4 raw paths bit-exact; fp16 and
group-wise (dequantised) outputs within 1e-2 relative Frobenius error and
2e-2 max-abs relative error (max|got-ref| / max|ref|).
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MANIFEST = json.load(open(os.path.join(GOLD, "manifest.json")))
REL_FRO = 1e-2
MAX_ABS_REL = 2e-2


def close_enough(orc, got, ref):
    fro, mar = orc.rel_frobenius(got, ref), orc.max_abs_rel(got, ref)
    assert fro <= REL_FRO and mar <= MAX_ABS_REL, (fro, mar)
    return fro, mar


# ---------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_golden_fixture(rkb, dev, orc, name):
    meta = MANIFEST[name]
    z = np.load(os.path.join(GOLD, name + ".npz"))
    A, B, exp = z["A"], z["B"], z["C"]
    M, K, N, g = meta["M"], meta["K"], meta["N"], meta["group"]
    kind = meta["kind"]
    if kind == "int8":
        C = np.full((M, N), -0x55555556, np.int32)
        assert dev.matmul_int8(M, K, N, A, B, C) == 0
        assert np.array_equal(C, exp)
    elif kind == "int4":
        C = np.zeros((M, N), np.int32)
        assert dev.matmul_int4(M, K, N, A, B, C) == 0
        assert np.array_equal(C, exp)
    elif kind == "fp16":
        C = np.zeros((M, N), np.float16)
        assert dev.matmul_fp16(M, K, N, A, B, C) == 0
        # integer-valued inputs (the gate draws rand()%3): every partial sum is
        # exact in fp32, so the result is bit-identical whatever the order
        assert np.array_equal(C.view(np.uint16), exp.view(np.uint16))
    else:
        C = np.zeros((M, N), np.float32)
        f = dev.matmul_int8_groupwise if kind == "int8_gw" else dev.matmul_int4_groupwise
        assert f(M, K, N, A, B, z["a_scale"], z["b_scale"], C, g) == 0
        close_enough(orc, C, exp)


# ---------------------------------------------------------------- int8 raw: bit-exact
INT8_SHAPES = [(1, 32, 32), (4, 32, 32), (64, 512, 256), (12, 96, 64), (132, 96, 96),
               (300, 4096, 768), (128, 15360, 256), (260, 1024, 5888)]


@pytest.mark.parametrize("M,K,N", INT8_SHAPES)
def test_int8_exact_vs_oracle(dev, orc, M, K, N):
    A = orc.uniform_i8(M * 7 + K, -128, 127, (M, K))
    B = orc.uniform_i8(N * 13 + K, -128, 127, (N, K))
    C = np.full((M, N), 0x5A5A5A5A, np.int32)
    assert dev.matmul_int8(M, K, N, A, B, C) == 0
    assert np.array_equal(C, orc.matmul_int8(A, B, nthreads=8))


def test_int8_extreme_values_exact(dev, orc):
    # all -128 * -128 over K=15360: 251,658,240 per element -- exact in int32
    M, K, N = 128, 15360, 256
    A = np.full((M, K), -128, np.int8)
    B = np.full((N, K), -128, np.int8)
    C = np.zeros((M, N), np.int32)
    assert dev.matmul_int8(M, K, N, A, B, C) == 0
    assert (C == 128 * 128 * K).all()


def test_int8_device_pointers_match_host(dev, orc):
    import torch
    M, K, N = 512, 3840, 1024
    A = orc.uniform_i8(11, -128, 127, (M, K))
    B = orc.uniform_i8(12, -128, 127, (N, K))
    Ch = np.zeros((M, N), np.int32)
    assert dev.matmul_int8(M, K, N, A, B, Ch) == 0
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    assert dev.matmul_int8(M, K, N, dA, dB, dC) == 0
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy(), Ch)


def test_int8_output_coverage_and_guards(dev, orc):
    """Every output element written, nothing written outside C (sentinels)."""
    import torch
    M, K, N = 200, 256, 320
    A = orc.uniform_i8(21, -128, 127, (M, K))
    B = orc.uniform_i8(22, -128, 127, (N, K))
    guard = 4096
    buf = torch.full((M * N + 2 * guard,), -0x55555556, dtype=torch.int32, device="cuda")
    C = buf[guard:guard + M * N]
    assert dev.matmul_int8(M, K, N, torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), C) == 0
    torch.cuda.synchronize()
    b = buf.cpu().numpy()
    assert (b[:guard] == -0x55555556).all() and (b[-guard:] == -0x55555556).all()
    assert np.array_equal(b[guard:-guard].reshape(M, N), orc.matmul_int8(A, B))


def test_int8_large_prefill_rows_sampled(dev, orc):
    """Config-5 gate+up shape, device resident; exact on sampled rows incl. tile edges."""
    import torch
    M, K, N = 4096, 3840, 5888
    A = orc.uniform_i8(31, -127, 127, (M, K))
    B = orc.uniform_i8(32, -127, 127, (N, K))
    dC = torch.empty((M, N), dtype=torch.int32, device="cuda")
    assert dev.matmul_int8(M, K, N, torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), dC) == 0
    C = dC.cpu().numpy()
    rows = [0, 1, 127, 128, 129, 2047, 2048, 4094, 4095]
    ref = orc.matmul_int8(A[rows], B, nthreads=8)
    assert np.array_equal(C[rows], ref)


# ---------------------------------------------------------------- int4 raw: bit-exact
@pytest.mark.parametrize("M,K,N", [(4, 32, 64), (64, 512, 256), (100, 3840, 640)])
def test_int4_exact_vs_oracle(dev, orc, M, K, N):
    A = orc.uniform_i8(M + 1, -8, 7, (M, K))
    B = orc.uniform_i8(N + 2, -8, 7, (N, K))
    C = np.zeros((M, N), np.int32)
    assert dev.matmul_int4(M, K, N, A, B, C) == 0
    assert np.array_equal(C, orc.matmul_int8(A, B))


# ---------------------------------------------------------------- fp16
@pytest.mark.parametrize("M,K,N", [(1, 64, 48), (4, 32, 16), (64, 512, 256), (260, 4096, 4096)])
def test_fp16_vs_oracle(dev, orc, M, K, N):
    A = orc.normal_f16(M + K, 1.0 / np.sqrt(K), (M, K))
    B = orc.normal_f16(N + K + 1, 1.0, (N, K))
    C = np.zeros((M, N), np.float16)
    assert dev.matmul_fp16(M, K, N, A, B, C) == 0
    R, C16 = orc.matmul_fp16(A, B, nthreads=8)
    fro, mar = close_enough(orc, C.astype(np.float32), R)
    assert fro < 1e-3   # fp32 accumulate: only the final fp16 rounding remains


def test_fp16_config2_device(dev, orc):
    """Config 2: M=512 K=4096 N=4096, N(0,1)/sqrt(K) inputs, sampled rows."""
    import torch
    M, K, N = 512, 4096, 4096
    A = orc.normal_f16(41, 1.0 / np.sqrt(K), (M, K))
    B = orc.normal_f16(42, 1.0 / np.sqrt(K), (N, K))
    dC = torch.empty((M, N), dtype=torch.float16, device="cuda")
    assert dev.matmul_fp16(M, K, N, torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), dC) == 0
    C = dC.cpu().numpy()
    rows = list(range(0, M, 37)) + [M - 1]
    R, _ = orc.matmul_fp16(A[rows], B, nthreads=8)
    close_enough(orc, C[rows].astype(np.float32), R)


# ---------------------------------------------------------------- group-wise
@pytest.mark.parametrize("bits,M,K,N,group,rowconst", [
    (8, 32, 576, 64, 96, False), (8, 64, 3840, 256, 32, True), (4, 64, 512, 128, 128, False),
    (4, 128, 3840, 512, 32, True), (4, 4, 64, 64, 32, False)])
def test_groupwise_vs_oracle(dev, orc, bits, M, K, N, group, rowconst):
    lo, hi = (-8, 7) if bits == 4 else (-127, 127)
    nG = K // group
    A = orc.uniform_i8(M + 5, -127, 127, (M, K))
    B = orc.uniform_i8(N + 6, lo, hi, (N, K))
    if rowconst:
        a = np.repeat(orc.uniform_f32(7, 0.01, 0.05, (M, 1)), nG, axis=1)
    else:
        a = orc.uniform_f32(7, 0.5, 1.5, (M, nG))
    b = orc.uniform_f32(8, 0.005, 0.02, (N, nG))
    C = np.zeros((M, N), np.float32)
    f = dev.matmul_int4_groupwise if bits == 4 else dev.matmul_int8_groupwise
    assert f(M, K, N, A, B, a, b, C, group) == 0
    close_enough(orc, C, orc.gw_ref(A, B, a, b, group, nthreads=8))


def test_groupwise_config3_rows_sampled(rkb, dev, orc):
    """Config 3 (W4A8 at 12B prefill) through the resident int4 group-wise path."""
    import ctypes
    import torch
    M, K, N, group = 2048, 3840, 15360, 32
    nG = K // group
    A = orc.uniform_i8(51, -127, 127, (M, K))
    B = orc.uniform_i8(52, -8, 7, (N, K))
    a = np.repeat(orc.uniform_f32(53, 0.01, 0.05, (M, 1)), nG, axis=1).astype(np.float32)
    b = orc.uniform_f32(54, 0.005, 0.02, (N, nG))
    ctx = rkb.lib.rocket_i4_ctx_create(1)
    assert ctx
    w = rkb.lib.rocket_i4_weights_pack_gw(ctx, M, K, N, rkb.ptr(B), group)
    assert w
    assert rkb.lib.rocket_i4_weights_bytes(w) >= N * K // 2
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    rc = rkb.lib.rocket_matmul_int4_prepacked_gw(ctx, M, K, N, rkb.ptr(A), rkb.ptr(a), rkb.ptr(b),
                                                 rkb.ptr(dC), w)
    rkb.lib.rocket_i4_weights_free(ctx, w)
    rkb.lib.rocket_i4_ctx_free(ctx)
    assert rc == 0
    C = dC.cpu().numpy()
    rows = [0, 127, 128, 1000, 2047]
    close_enough(orc, C[rows], orc.gw_ref(A[rows], B, a[rows], b, group, nthreads=8))


@pytest.mark.parametrize("M,K,N", [(512, 4096, 4096), (260, 8192, 1024), (64, 4096, 2048)])
def test_fp16_small_m_split_k(dev, orc, M, K, N, monkeypatch):
    """The opt-in split-K CTA-pair path (fp32 partials reduced in a fixed order):
    results stay within the fp16 bound and are deterministic."""
    import torch
    monkeypatch.setenv("ROCKET_GEMM_SPLITK", "3")
    A = orc.normal_f16(M + 3, 1.0 / np.sqrt(K), (M, K))
    B = orc.normal_f16(N + 4, 1.0, (N, K))
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C1 = torch.empty((M, N), dtype=torch.float16, device="cuda")
    C2 = torch.empty_like(C1)
    assert dev.matmul_fp16(M, K, N, dA, dB, C1) == 0
    assert dev.matmul_fp16(M, K, N, dA, dB, C2) == 0
    torch.cuda.synchronize()
    assert torch.equal(C1, C2)
    rows = list(range(0, M, max(1, M // 16))) + [M - 1]
    R, _ = orc.matmul_fp16(A[rows], B, nthreads=8)
    close_enough(orc, C1.cpu().numpy()[rows].astype(np.float32), R)


# ---------------------------------------------------------------- stream-K tail
# When CTA-pair tiles leave the last wave under-filled, int8 GEMMs may run the
# stream-K tail: the tail tiles' K-blocks are split over all SM pairs, every
# segment adds its int32 accumulator into the tile's zeroed sum buffer, and the
# last segment to arrive stores C.  Exact in any arrival order.  The policy is
# forced here (rocket_b200_gemm_policy) so small shapes take that path too.
@pytest.fixture
def force_sk(rkb):
    def force(variant):
        assert rkb.lib.rocket_b200_gemm_policy(variant, 1) == 0
    yield force
    rkb.lib.rocket_b200_gemm_policy(0, -1)


@pytest.mark.parametrize("variant,M,K,N", [(512, 1000, 1024, 3840),    # one partial wave: 60 tiles on 74 pairs
                                           (512, 2048, 2048, 3840),    # 1.62 waves
                                           (384, 900, 2048, 2016),     # ragged M and N edges, 256 x 128 tiles
                                           (512, 4096, 3840, 3840)])   # o_proj shape, 3.24 waves
def test_int8_stream_k_exact(rkb, dev, orc, force_sk, variant, M, K, N):
    force_sk(variant)
    A = orc.uniform_i8(M + 5, -127, 127, (M, K))
    B = orc.uniform_i8(N + 6, -127, 127, (N, K))
    C = np.full((M, N), -0x55555556, np.int32)
    for _ in range(2):      # the sum buffers must start from zero on every launch
        assert dev.matmul_int8(M, K, N, A, B, C) == 0
    assert np.array_equal(C, orc.matmul_int8(A, B, nthreads=16))


def test_int8_stream_k_down_shape_rows(dev, orc):
    """Config-5 down GEMM (4096 x 15360 x 3840) under the automatic policy, which
    takes the stream-K tail at this shape; exact on sampled rows."""
    import torch
    M, K, N = 4096, 15360, 3840
    A = orc.uniform_i8(41, -127, 127, (M, K))
    B = orc.uniform_i8(42, -127, 127, (N, K))
    dC = torch.empty((M, N), dtype=torch.int32, device="cuda")
    assert dev.matmul_int8(M, K, N, torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), dC) == 0
    C = dC.cpu().numpy()
    rows = [0, 1, 127, 128, 255, 256, 1000, 2047, 3583, 3584, 3840, 4095]
    assert np.array_equal(C[rows], orc.matmul_int8(A[rows], B, nthreads=16))


def test_gemm_policy_rejects_unknown_values(rkb):
    assert rkb.lib.rocket_b200_gemm_policy(320, -1) != 0
    assert rkb.lib.rocket_b200_gemm_policy(0, 2) != 0
    assert rkb.lib.rocket_b200_gemm_policy(0, -1) == 0


@pytest.mark.parametrize("M,K,N", [(1000, 1024, 3840), (900, 2048, 2016)])
def test_fp16_pair_tiles_ragged(rkb, dev, orc, M, K, N):
    """fp16 / fp32-out through the pair kernel with ragged M / N edges (fp16 never
    takes stream-K: float sums would depend on arrival order)."""
    A = orc.normal_f16(M + 7, 1.0 / np.sqrt(K), (M, K))
    B = orc.normal_f16(N + 8, 1.0, (N, K))
    C = np.zeros((M, N), np.float16)
    assert dev.matmul_fp16(M, K, N, A, B, C) == 0
    R, _ = orc.matmul_fp16(A, B, nthreads=16)
    fro, mar = close_enough(orc, C.astype(np.float32), R)
    assert fro < 1e-3
    import ctypes
    C32 = np.zeros((M, N), np.float32)
    assert rkb.lib.rocket_matmul_fp16_f32out(dev.fd, M, K, N, ctypes.c_void_p(A.ctypes.data),
                                             ctypes.c_void_p(B.ctypes.data), ctypes.c_void_p(C32.ctypes.data)) == 0
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    assert np.max(np.abs(C32 - ref)) <= 1e-4 * np.max(np.abs(ref))
