"""GPU parity of the precise group-wise mode (the default) against the
reference's definition and its own gate bound.

The reference computes group-wise products as exact integer partials per K
group, scaled by a_scale[m,g] * b_scale[n,g] and summed in fp32
(src/rocket_matmul.c:2842-2856, src/rocket_prepacked_int8.c:620-632).  Its
gates compare against an fp64 evaluation with max|got - ref| <= 1e-5 * rms(ref)
(tests/matmul_int8_groupwise_rocket.c:59-82) -- the bound used here.  The int4
gates additionally count an element bad when its relative error exceeds 1e-4
AND its absolute error exceeds 1e-2 (tests/matmul_int4_groupwise_rocket.c:79-82).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RMS_TOL = 1e-5


def check_gate(orc, got, ref, int4=False):
    err = orc.rms_normalised_err(got, ref)
    assert np.isfinite(got).all()
    assert err <= RMS_TOL, err
    if int4:
        ad = np.abs(got.astype(np.float64) - ref)
        rd = ad / (np.abs(ref) + 1e-6)
        assert not np.any((rd > 1e-4) & (ad > 1e-2))
    return err


@pytest.fixture(autouse=True)
def precise_mode(rkb):
    assert rkb.lib.rocket_b200_gw_mode(0) == 0
    yield
    rkb.lib.rocket_b200_gw_mode(0)


# the reference gate's own shape and group sweep (matmul_int8_groupwise_rocket.c main)
@pytest.mark.parametrize("group", [96, 288, 576, 1440, 2880])
def test_int8_gate_groups(dev, orc, group):
    M, K, N = 128, 2880, 256
    nG = K // group
    A = orc.uniform_i8(11, -127, 127, (M, K))
    B = orc.uniform_i8(12, -127, 127, (N, K))
    a = orc.uniform_f32(13, 0.5, 1.5, (M, nG))
    b = orc.uniform_f32(14, 0.5, 1.5, (N, nG))
    C = np.zeros((M, N), np.float32)
    assert dev.matmul_int8_groupwise(M, K, N, A, B, a, b, C, group) == 0
    check_gate(orc, C, orc.gw_ref(A, B, a, b, group, nthreads=8))


@pytest.mark.parametrize("bits,M,K,N,group,rowconst", [
    (4, 128, 3840, 256, 128, False),     # int4 gate default
    (4, 4, 64, 64, 32, False),
    (4, 132, 96, 320, 32, True),         # partial 64-wide K block, M and N tails
    (4, 256, 3840, 512, 32, True),       # config-3 group and per-row activation scale
    (8, 4, 96, 32, 32, False),
    (8, 260, 2048, 96, 2048, False),     # int8 group 2048: one int32 partial, converted once
    (8, 64, 3840, 256, 32, True),
])
def test_precise_vs_fp64(dev, orc, bits, M, K, N, group, rowconst):
    lo, hi = (-8, 7) if bits == 4 else (-127, 127)
    nG = K // group
    A = orc.uniform_i8(M + 21, -127, 127, (M, K))
    B = orc.uniform_i8(N + 22, lo, hi, (N, K))
    if rowconst:
        a = np.repeat(orc.uniform_f32(23, 0.01, 0.05, (M, 1)), nG, axis=1)
    else:
        a = orc.uniform_f32(23, 0.5, 1.5, (M, nG))
    b = orc.uniform_f32(24, 0.005, 0.02, (N, nG))
    C = np.zeros((M, N), np.float32)
    f = dev.matmul_int4_groupwise if bits == 4 else dev.matmul_int8_groupwise
    assert f(M, K, N, A, B, a, b, C, group) == 0
    check_gate(orc, C, orc.gw_ref(A, B, a, b, group, nthreads=8), int4=bits == 4)


def test_int8_extreme_partials_exact(dev, orc):
    """|a w| = 2^14 everywhere: a 1024-wide partial reaches 2^24, the edge of
    fp32's exact integer range.  With one group and unit scales the output IS
    the partial, so it must equal the integer product exactly."""
    M, K, N, group = 64, 1024, 64, 1024
    a = np.ones((M, 1), np.float32)
    b = np.ones((N, 1), np.float32)
    A = np.full((M, K), -128, np.int8)
    B = np.full((N, K), -128, np.int8)
    C = np.zeros((M, N), np.float32)
    assert dev.matmul_int8_groupwise(M, K, N, A, B, a, b, C, group) == 0
    assert np.all(C == np.float32(2.0 ** 24))
    rng = np.random.default_rng(5)
    A = np.where(rng.random((M, K)) < 0.5, -128, 127).astype(np.int8)
    B = np.where(rng.random((N, K)) < 0.5, -128, 127).astype(np.int8)
    assert dev.matmul_int8_groupwise(M, K, N, A, B, a, b, C, group) == 0
    assert np.array_equal(C.astype(np.int64), A.astype(np.int64) @ B.astype(np.int64).T)


@pytest.mark.parametrize("bits,group", [(8, 224), (8, 256), (4, 640)])
def test_partial_extremes_exact(dev, bits, group):
    """Extreme codes with one group and unit scales: C is the int32 partial
    converted to fp32, so it must equal the integer product exactly (every
    |P| here is at most 2^22).  int8 groups 224 and 256, and the widest int4
    group the entry accepts (640)."""
    M, N, K = 64, 64, group
    lo, hi = (-8, 7) if bits == 4 else (-128, 127)
    rng = np.random.default_rng(group + bits)
    a = np.ones((M, 1), np.float32)
    b = np.ones((N, 1), np.float32)
    f = dev.matmul_int4_groupwise if bits == 4 else dev.matmul_int8_groupwise
    for A, B in ((np.full((M, K), -128, np.int8), np.full((N, K), lo, np.int8)),
                 (np.where(rng.random((M, K)) < 0.5, -128, 127).astype(np.int8),
                  np.where(rng.random((N, K)) < 0.5, lo, hi).astype(np.int8))):
        C = np.zeros((M, N), np.float32)
        assert f(M, K, N, A, B, a, b, C, group) == 0
        assert np.array_equal(C.astype(np.int64), A.astype(np.int64) @ B.astype(np.int64).T)


def test_int8_wide_group(dev, orc):
    """A 2048-wide int8 group is one int32 partial (up to 2^25 in magnitude
    here, so its conversion to fp32 rounds once, as the reference's does)."""
    M, K, N, group = 64, 4096, 64, 2048
    nG = K // group
    rng = np.random.default_rng(6)
    A = np.where(rng.random((M, K)) < 0.5, -128, 127).astype(np.int8)
    B = np.where(rng.random((N, K)) < 0.5, -128, 127).astype(np.int8)
    a = orc.uniform_f32(41, 0.5, 1.5, (M, nG))
    b = orc.uniform_f32(42, 0.5, 1.5, (N, nG))
    C = np.zeros((M, N), np.float32)
    assert dev.matmul_int8_groupwise(M, K, N, A, B, a, b, C, group) == 0
    check_gate(orc, C, orc.gw_ref(A, B, a, b, group, nthreads=8))


def test_fast_mode_switch(rkb, dev, orc):
    """Mode 1 (w * scale rounded to fp16) stays within the north-star bound and
    differs from the precise mode; mode 0 comes back bit-identical."""
    M, K, N, group = 64, 1024, 256, 32
    nG = K // group
    A = orc.uniform_i8(31, -127, 127, (M, K))
    B = orc.uniform_i8(32, -8, 7, (N, K))
    a = orc.uniform_f32(33, 0.5, 1.5, (M, nG))
    b = orc.uniform_f32(34, 0.005, 0.02, (N, nG))
    ref = orc.gw_ref(A, B, a, b, group, nthreads=8)
    P = np.zeros((M, N), np.float32)
    assert dev.matmul_int4_groupwise(M, K, N, A, B, a, b, P, group) == 0
    assert rkb.lib.rocket_b200_gw_mode(1) == 0
    F = np.zeros((M, N), np.float32)
    assert dev.matmul_int4_groupwise(M, K, N, A, B, a, b, F, group) == 0
    assert rkb.lib.rocket_b200_gw_mode(0) == 0
    P2 = np.zeros((M, N), np.float32)
    assert dev.matmul_int4_groupwise(M, K, N, A, B, a, b, P2, group) == 0
    assert orc.rel_frobenius(F, ref) <= 1e-2 and orc.max_abs_rel(F, ref) <= 2e-2
    assert orc.rms_normalised_err(P, ref) < orc.rms_normalised_err(F, ref)
    assert np.array_equal(P, P2)
    assert rkb.lib.rocket_b200_gw_mode(2) == rkb.ROCKET_E_SHAPE


def test_config3_resident_precise_rows_sampled(rkb, orc):
    """Config 3 (W4A8, 2048 x 3840 x 15360, group 32) through the resident int4
    group-wise entry, held to the gate's 1e-5 * rms bound on sampled rows."""
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
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    rc = rkb.lib.rocket_matmul_int4_prepacked_gw(ctx, M, K, N, rkb.ptr(A), rkb.ptr(a), rkb.ptr(b),
                                                 rkb.ptr(dC), w)
    rkb.lib.rocket_i4_weights_free(ctx, w)
    rkb.lib.rocket_i4_ctx_free(ctx)
    assert rc == 0
    C = dC.cpu().numpy()
    rows = [0, 1, 127, 128, 1000, 2047]
    check_gate(orc, C[rows], orc.gw_ref(A[rows], B, a[rows], b, group, nthreads=8), int4=True)
