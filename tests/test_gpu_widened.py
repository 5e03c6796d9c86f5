"""GPU parity of the widened entries through the C ABI: fp16 -> fp32 output,
bf16 / tf32 one-shots, exact int16, the batched and streaming fp16 matmuls,
bf16 multi-thread / stream, and the reduction family.

Tolerances (each stated beside its check):
  exact int16 ............ bit-exact (int64)
  fp16 -> fp32, bf16 ..... max|got-ref| <= 1e-4 * max|ref|: fp32 accumulation of
                           exact products against an fp64 sum
  tf32 ................... normalised error < 2e-3 (the reference gate's bound;
                           tf32 keeps 10 mantissa bits of each input)
  batch / stream ......... bit-identical to the one-shot fp16 entry
  reductions ............. fp32 accumulation against the reference's fp64 loop:
                           cumsum within one fp16 ulp (+1e-4 of the row
                           scale for cancellations), scale_rows bit-exact,
                           reduce 5e-5 of sum|x|, CE 1e-3 relative
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def P(a):
    return ctypes.c_void_p(a.ctypes.data)


def arr_of_ptrs(arrs):
    return (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def max_rel(got, ref):
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))


def fp16_inputs(orc, M, K, N, seed=0):
    A = orc.normal_f16(seed + 11, 1.0 / np.sqrt(K), (M, K))
    B = orc.normal_f16(seed + 12, 1.0, (N, K))
    return A, B


@pytest.mark.parametrize("M,K,N", [(1, 64, 48), (64, 4096, 512), (260, 1024, 528)])
def test_fp16_f32out(rkb, dev, orc, M, K, N):
    A, B = fp16_inputs(orc, M, K, N)
    C = np.full((M, N), np.nan, np.float32)
    assert rkb.lib.rocket_matmul_fp16_f32out(dev.fd, M, K, N, P(A), P(B), P(C)) == 0
    assert max_rel(C, orc.matmul_f64(A, B)) <= 1e-4


@pytest.mark.parametrize("M,K,N", [(1, 512, 256), (512, 3840, 4096), (68, 96, 144)])
def test_bf16(rkb, dev, orc, M, K, N):
    A = orc.normal_f32(21, 0.0, 1.0, (M, K))
    B = orc.normal_f32(22, 0.0, 1.0, (N, K))
    C = np.full((M, N), np.nan, np.float32)
    assert rkb.lib.rocket_matmul_bf16(dev.fd, M, K, N, P(A), P(B), P(C)) == 0
    assert max_rel(C, orc.matmul_bf16(A, B)) <= 1e-4


@pytest.mark.parametrize("M,K,N", [(4, 16, 16), (68, 272, 144), (512, 3840, 4096)])
def test_tf32(rkb, dev, orc, M, K, N):
    A = orc.normal_f32(31, 0.0, 1.0, (M, K))
    B = orc.normal_f32(32, 0.0, 1.0, (N, K))
    C = np.full((M, N), np.nan, np.float32)
    assert rkb.lib.rocket_matmul_tf32(dev.fd, M, K, N, P(A), P(B), P(C)) == 0
    R = orc.matmul_f64(A, B)
    assert np.isfinite(C).all()
    assert max_rel(C, R) < 2e-3


@pytest.mark.parametrize("M,K,N", [(1, 64, 32), (256, 1024, 512), (132, 4096, 96)])
def test_int16_exact(rkb, dev, orc, M, K, N):
    rng = np.random.default_rng(M * 7 + K)
    A = rng.integers(-32768, 32768, (M, K), dtype=np.int16)
    B = rng.integers(-32768, 32768, (N, K), dtype=np.int16)
    A.flat[:3] = [-32768, 32767, 32639]          # both ends of the range and the clamp edge
    B.flat[:3] = [32767, -32768, -1]
    C = np.zeros((M, N), np.int64)
    assert rkb.lib.rocket_matmul_int16_exact(dev.fd, M, K, N, P(A), P(B), P(C)) == 0
    assert np.array_equal(C, orc.matmul_int16_exact(A, B))


def test_fp16_batch_and_handle_match_one_shot(rkb, dev, orc):
    M, K, N, nb = 256, 256, 528, 5
    As = [orc.normal_f16(40 + i, 0.1, (M, K)) for i in range(nb)]
    Bs = [orc.normal_f16(50 + i, 1.0, (N, K)) for i in range(nb)]
    ref = []
    for a, b in zip(As, Bs):
        c = np.zeros((M, N), np.float16)
        assert dev.matmul_fp16(M, K, N, a, b, c) == 0
        ref.append(c)
    Cs = [np.zeros((M, N), np.float16) for _ in range(nb)]
    assert rkb.lib.rocket_matmul_fp16_batch(dev.fd, M, K, N, nb, arr_of_ptrs(As), arr_of_ptrs(Bs),
                                            arr_of_ptrs(Cs)) == 0
    assert all(np.array_equal(c, r) for c, r in zip(Cs, ref))
    h = rkb.lib.rocket_mm_batch_create(dev.fd)
    assert h
    Cs2 = [np.zeros((M, N), np.float16) for _ in range(nb)]
    try:
        assert rkb.lib.rocket_mm_batch_run(h, M, K, N, nb, arr_of_ptrs(As), arr_of_ptrs(Bs),
                                           arr_of_ptrs(Cs2)) == 0
    finally:
        rkb.lib.rocket_mm_batch_free(h)
    assert all(np.array_equal(c, r) for c, r in zip(Cs2, ref))


def test_fp16_stream_and_fused_match_one_shot(rkb, dev, orc):
    M, K = 128, 1024
    Ns = [512, 256, 96]
    A = orc.normal_f16(60, 1.0 / 32, (M, K))
    Bs = [orc.normal_f16(61 + i, 1.0, (n, K)) for i, n in enumerate(Ns)]
    Bcat = np.concatenate(Bs, axis=0)
    ref = np.zeros((M, sum(Ns)), np.float16)
    assert dev.matmul_fp16(M, K, sum(Ns), A, Bcat, ref) == 0
    s = rkb.lib.rocket_stream_create(2)
    assert s
    try:
        C = np.zeros((M, Ns[0]), np.float16)
        for _ in range(2):      # second call reuses the stream's resident buffers
            assert rkb.lib.rocket_matmul_fp16_stream(s, M, K, Ns[0], P(A), P(Bs[0]), P(C)) == 0
            assert np.array_equal(C, ref[:, :Ns[0]])
        Cf = np.zeros((M, sum(Ns)), np.float16)
        ns = (ctypes.c_int * 3)(*Ns)
        assert rkb.lib.rocket_matmul_fp16_stream_fused(s, M, K, arr_of_ptrs(Bs), ns, 3, P(A), P(Cf)) == 0
        assert np.array_equal(Cf, ref)
    finally:
        rkb.lib.rocket_stream_free(s)


def test_bf16_mt_and_stream_bit_identical(rkb, dev, orc):
    M, K, N = 512, 3840, 4096
    A = orc.normal_f32(70, 0.0, 1.0, (M, K))
    B = orc.normal_f32(71, 0.0, 1.0, (N, K))
    Cr = np.zeros((M, N), np.float32)
    assert rkb.lib.rocket_matmul_bf16(dev.fd, M, K, N, P(A), P(B), P(Cr)) == 0
    Cm = np.zeros_like(Cr)
    assert rkb.lib.rocket_matmul_bf16_mt(M, K, N, P(A), P(B), P(Cm), 4) == 0
    assert np.array_equal(Cm, Cr)
    for nt in (1, 4):
        s = rkb.lib.rocket_bf16_stream_create(nt)
        assert s
        try:
            Cs = np.zeros_like(Cr)
            assert rkb.lib.rocket_matmul_bf16_stream(s, M, K, N, P(A), P(B), P(Cs)) == 0
            assert np.array_equal(Cs, Cr)
        finally:
            rkb.lib.rocket_bf16_stream_free(s)


def fp16_close(got, ref, scale):
    got = np.asarray(got, np.float64)
    refd = np.asarray(ref, np.float64)
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64)
    return bool(np.all(np.abs(got - refd) <= ulp + 1e-4 * scale[:, None]))


@pytest.mark.parametrize("M,N", [(37, 300), (1, 1), (512, 4096), (3, 70000)])
def test_cumsum(rkb, dev, orc, M, N):
    x = orc.normal_f16(80 + N, 1.0, (M, N))
    for exc in (0, 1):
        for rev in (0, 1):
            y = np.zeros((M, N), np.float16)
            assert rkb.lib.rocket_cumsum_fp16(dev.fd, M, N, P(x), P(y), exc, rev) == 0
            ref = orc.cumsum(x, exc, rev)
            scale = np.max(np.abs(ref.astype(np.float64)), axis=1) + 1.0
            assert fp16_close(y, ref, scale), (exc, rev)


@pytest.mark.parametrize("M,H", [(37, 300), (1, 1), (4096, 4096), (2, 100000)])
def test_reduce_feature(rkb, dev, orc, M, H):
    x = orc.normal_f16(90 + H, 1.0, (M, H))
    for mean in (0, 1):
        o = np.zeros(M, np.float32)
        assert rkb.lib.rocket_reduce_feature_fp16(dev.fd, M, H, P(x), P(o), mean) == 0
        ref = orc.reduce_feature(x, mean)
        absum = np.abs(x.astype(np.float64)).sum(axis=1) / (H if mean else 1)
        assert np.all(np.abs(o - ref) <= 5e-5 * absum + 1e-7)


@pytest.mark.parametrize("M,N", [(37, 300), (1, 8), (1024, 4096)])
def test_scale_rows(rkb, dev, orc, M, N):
    x = orc.normal_f16(100 + N, 1.0, (M, N))
    r = orc.uniform_f32(101, -2.0, 2.0, (M,))
    y = np.zeros((M, N), np.float16)
    assert rkb.lib.rocket_scale_rows_fp16(dev.fd, M, N, P(x), P(r), P(y)) == 0
    assert np.array_equal(y.view(np.uint16), orc.scale_rows(x, r).view(np.uint16))


@pytest.mark.parametrize("M,N", [(33, 1000), (1, 1), (64, 32000), (4, 150000)])
def test_cross_entropy(rkb, dev, orc, M, N):
    x = orc.normal_f16(110 + N, 3.0, (M, N))
    t = ((np.arange(M) * 7919) % N).astype(np.int32)
    if M > 2:
        t[0], t[1] = -1, N      # out-of-range targets contribute no logit term
    loss = np.zeros(M, np.float32)
    assert rkb.lib.rocket_cross_entropy_fp16(dev.fd, M, N, P(x), P(t), P(loss)) == 0
    ref = orc.cross_entropy(x, t)
    assert np.all(np.abs(loss - ref) <= 1e-3 * np.maximum(1.0, np.abs(ref)))


def test_golden_reductions(rkb, dev, orc):
    import os
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reduce_golden.npz"))
    gi = orc.reduce_golden_inputs()
    x = gi["x"]
    M, N = x.shape
    y = np.zeros_like(x)
    assert rkb.lib.rocket_scale_rows_fp16(dev.fd, M, N, P(x), P(gi["r"]), P(y)) == 0
    assert np.array_equal(y.view(np.uint16), g["scale"].view(np.uint16))
    lg, t = gi["logits"], gi["target"]
    loss = np.zeros(lg.shape[0], np.float32)
    assert rkb.lib.rocket_cross_entropy_fp16(dev.fd, lg.shape[0], lg.shape[1], P(lg), P(t), P(loss)) == 0
    assert np.all(np.abs(loss - g["ce"]) <= 1e-3 * np.maximum(1.0, np.abs(g["ce"])))
