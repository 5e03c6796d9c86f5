"""GPU: resident-weight contexts and the N-split fan-out.

Mirrors the reference's resident gates (tests/matmul_int8_prepacked_rocket.c,
matmul_int4_prepacked_rocket.c, matmul_int4_prepacked_gw_rocket.c,
matmul_mt_rocket.c): resident == one-shot bit-exact, several distinct
weights on one ctx do not alias, a weight packed at one M serves another M,
and every worker count gives the same answer.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _i8(rkb, orc, nthreads, M, K, N, W=3, Ms=None):
    ctx = rkb.lib.rocket_i8_ctx_create(nthreads)
    assert ctx
    A = orc.uniform_i8(100 + M, -128, 127, (M, K))
    Bs = [orc.uniform_i8(200 + w, -128, 127, (N, K)) for w in range(W)]
    ws = [rkb.lib.rocket_i8_weights_pack(ctx, M, K, N, rkb.ptr(B)) for B in Bs]
    assert all(ws)
    try:
        for B, w in zip(Bs, ws):
            for m in (Ms or [M]):
                C = np.zeros((m, N), np.int32)
                assert rkb.lib.rocket_matmul_int8_prepacked(ctx, m, K, N, rkb.ptr(A[:m].copy()), rkb.ptr(C), w) == 0
                assert np.array_equal(C, orc.matmul_int8(A[:m], B, nthreads=8))
        # reuse the first weight after the others were packed (aliasing guard)
        C = np.zeros((M, N), np.int32)
        assert rkb.lib.rocket_matmul_int8_prepacked(ctx, M, K, N, rkb.ptr(A), rkb.ptr(C), ws[0]) == 0
        assert np.array_equal(C, orc.matmul_int8(A, Bs[0], nthreads=8))
        assert rkb.lib.rocket_i8_weights_bytes(ws[0]) == N * K
    finally:
        for w in ws:
            rkb.lib.rocket_i8_weights_free(ctx, w)
        rkb.lib.rocket_i8_ctx_free(ctx)


@pytest.mark.parametrize("nthreads", [1, 3, 5])
def test_i8_resident(rkb, dev, orc, nthreads):
    _i8(rkb, orc, nthreads, 64, 512, 320, W=3, Ms=[64, 4, 32])


def test_i8_resident_shape_mismatch(rkb, dev, orc):
    ctx = rkb.lib.rocket_i8_ctx_create(1)
    B = orc.uniform_i8(1, -128, 127, (64, 256))
    w = rkb.lib.rocket_i8_weights_pack(ctx, 32, 256, 64, rkb.ptr(B))
    A = np.zeros((32, 256), np.int8)
    C = np.zeros((32, 64), np.int32)
    assert rkb.lib.rocket_matmul_int8_prepacked(ctx, 32, 512, 64, rkb.ptr(A), rkb.ptr(C), w) == rkb.ROCKET_E_SHAPE
    assert rkb.lib.rocket_matmul_int8_prepacked(ctx, 6, 256, 64, rkb.ptr(A), rkb.ptr(C), w) == rkb.ROCKET_E_SHAPE
    # per-channel weight used on the group-wise entry
    f = np.ones(32 * 8, np.float32)
    Cf = np.zeros((32, 64), np.float32)
    assert rkb.lib.rocket_matmul_int8_prepacked_gw(ctx, 32, 256, 64, rkb.ptr(A), rkb.ptr(f), rkb.ptr(f),
                                                   rkb.ptr(Cf), w) == rkb.ROCKET_E_SHAPE
    rkb.lib.rocket_i8_weights_free(ctx, w)
    rkb.lib.rocket_i8_ctx_free(ctx)


@pytest.mark.parametrize("nthreads", [1, 2])
def test_i4_resident_matches_oneshot(rkb, dev, orc, nthreads):
    M, K, N = 96, 3840, 384
    ctx = rkb.lib.rocket_i4_ctx_create(nthreads)
    A = orc.uniform_i8(5, -8, 7, (M, K))
    B = orc.uniform_i8(6, -8, 7, (N, K))
    w = rkb.lib.rocket_i4_weights_pack(ctx, M, K, N, rkb.ptr(B))
    assert w
    # nibble-packed on the device: half the int8 footprint
    assert rkb.lib.rocket_i4_weights_bytes(w) < N * K
    C = np.zeros((M, N), np.int32)
    assert rkb.lib.rocket_matmul_int4_prepacked(ctx, M, K, N, rkb.ptr(A), rkb.ptr(C), w) == 0
    C1 = np.zeros((M, N), np.int32)
    assert dev.matmul_int4(M, K, N, A, B, C1) == 0
    assert np.array_equal(C, C1)
    assert np.array_equal(C, orc.matmul_int8(A, B, nthreads=8))
    rkb.lib.rocket_i4_weights_free(ctx, w)
    rkb.lib.rocket_i4_ctx_free(ctx)


@pytest.mark.parametrize("bits,nthreads", [(4, 1), (4, 3), (8, 1), (8, 2)])
def test_gw_resident_matches_oneshot(rkb, dev, orc, bits, nthreads):
    M, K, N, group = 64, 1024, 512, 128
    nG = K // group
    lo, hi = (-8, 7) if bits == 4 else (-127, 127)
    A = orc.uniform_i8(7, -127, 127, (M, K))
    B = orc.uniform_i8(8, lo, hi, (N, K))
    a = orc.uniform_f32(9, 0.5, 1.5, (M, nG))
    b = orc.uniform_f32(10, 0.5, 1.5, (N, nG))
    if bits == 4:
        ctx = rkb.lib.rocket_i4_ctx_create(nthreads)
        w = rkb.lib.rocket_i4_weights_pack_gw(ctx, M, K, N, rkb.ptr(B), group)
        run, free_w, free_c = (rkb.lib.rocket_matmul_int4_prepacked_gw, rkb.lib.rocket_i4_weights_free,
                               rkb.lib.rocket_i4_ctx_free)
        one = dev.matmul_int4_groupwise
    else:
        ctx = rkb.lib.rocket_i8_ctx_create(nthreads)
        w = rkb.lib.rocket_i8_weights_pack_gw(ctx, M, K, N, rkb.ptr(B), group)
        run, free_w, free_c = (rkb.lib.rocket_matmul_int8_prepacked_gw, rkb.lib.rocket_i8_weights_free,
                               rkb.lib.rocket_i8_ctx_free)
        one = dev.matmul_int8_groupwise
    assert ctx and w
    Cr = np.zeros((M, N), np.float32)
    assert run(ctx, M, K, N, rkb.ptr(A), rkb.ptr(a), rkb.ptr(b), rkb.ptr(Cr), w) == 0
    Co = np.zeros((M, N), np.float32)
    assert one(M, K, N, A, B, a, b, Co, group) == 0
    # same kernel, same per-element K order: resident == one-shot bit for bit
    assert np.array_equal(Cr, Co)
    ref = orc.gw_ref(A, B, a, b, group, nthreads=8)
    assert orc.rel_frobenius(Cr, ref) <= 1e-2 and orc.max_abs_rel(Cr, ref) <= 2e-2
    free_w(ctx, w)
    free_c(ctx)


def test_fp16_resident_and_mt(rkb, dev, orc):
    M, K, N = 128, 1024, 1040
    A = orc.normal_f16(1, 1.0 / 32, (M, K))
    B = orc.normal_f16(2, 1.0, (N, K))
    R, _ = orc.matmul_fp16(A, B, nthreads=8)
    C1 = np.zeros((M, N), np.float16)
    assert dev.matmul_fp16(M, K, N, A, B, C1) == 0
    for nt in (1, 2, 3, 4):
        C = np.zeros((M, N), np.float16)
        assert rkb.lib.rocket_matmul_fp16_mt(M, K, N, rkb.ptr(A), rkb.ptr(B), rkb.ptr(C), nt) == 0
        assert np.array_equal(C.view(np.uint16), C1.view(np.uint16)), nt
    ctx = rkb.lib.rocket_ctx_create(2)
    w = rkb.lib.rocket_weights_pack(ctx, M, K, N, rkb.ptr(B))
    assert w
    for m in (M, 4, 64):
        C = np.zeros((m, N), np.float16)
        assert rkb.lib.rocket_matmul_fp16_prepacked(ctx, m, K, N, rkb.ptr(A[:m].copy()), rkb.ptr(C), w) == 0
        assert np.array_equal(C.view(np.uint16), C1[:m].view(np.uint16))
    rkb.lib.rocket_weights_free(ctx, w)
    rkb.lib.rocket_ctx_free(ctx)
    fro = orc.rel_frobenius(C1.astype(np.float32), R)
    assert fro < 1e-3


def test_bo_roundtrip(rkb, dev):
    import ctypes

    class BO(ctypes.Structure):
        _fields_ = [("handle", ctypes.c_uint32), ("dma_address", ctypes.c_uint64),
                    ("mmap_offset", ctypes.c_uint64), ("size", ctypes.c_size_t), ("ptr", ctypes.c_void_p)]
    bo = BO()
    assert rkb.lib.rocket_bo_alloc(dev.fd, 10000, ctypes.byref(bo)) == 0
    assert bo.size >= 10000 and bo.ptr and bo.dma_address
    buf = (ctypes.c_uint8 * bo.size).from_address(bo.ptr)
    for i in range(bo.size):
        buf[i] = i & 0xFF
    assert rkb.lib.rocket_bo_fini(dev.fd, ctypes.byref(bo)) == 0
    for i in range(bo.size):
        buf[i] = 0
    assert rkb.lib.rocket_bo_prep(dev.fd, ctypes.byref(bo), 0, 2_000_000_000) == 0
    assert all(buf[i] == (i & 0xFF) for i in range(0, bo.size, 97))
    rkb.lib.rocket_bo_free(dev.fd, ctypes.byref(bo))


def test_async_enqueue_then_sync(rkb, dev, orc):
    """rocket_b200_set_async: device-resident resident calls queue without
    waiting; rocket_b200_ctx_sync returns their status; results unchanged."""
    import torch
    M, K, N = 256, 1024, 512
    ctx = rkb.lib.rocket_i8_ctx_create(1)
    A = orc.uniform_i8(61, -128, 127, (M, K))
    Bs = [orc.uniform_i8(62 + i, -128, 127, (N, K)) for i in range(3)]
    ws = [rkb.lib.rocket_i8_weights_pack(ctx, M, K, N, rkb.ptr(B)) for B in Bs]
    dA = torch.from_numpy(A).cuda()
    Cs = [torch.full((M, N), 7, dtype=torch.int32, device="cuda") for _ in Bs]
    rkb.lib.rocket_b200_set_async(1)
    try:
        for _ in range(3):
            for w, C in zip(ws, Cs):
                assert rkb.lib.rocket_matmul_int8_prepacked(ctx, M, K, N, rkb.ptr(dA), rkb.ptr(C), w) == 0
        assert rkb.lib.rocket_b200_ctx_sync(ctx) == 0
    finally:
        rkb.lib.rocket_b200_set_async(0)
    for B, C in zip(Bs, Cs):
        assert np.array_equal(C.cpu().numpy(), orc.matmul_int8(A, B, nthreads=8))
    for w in ws:
        rkb.lib.rocket_i8_weights_free(ctx, w)
    rkb.lib.rocket_i8_ctx_free(ctx)


# The bench's headline path: resident per-channel int8 at M = 4096 on the
# N-shard widths that one-rank-per-GPU runs use (QKV 5888, O 3840, gate+up
# 30720 at K 3840; down 3840 at K 15360; split over 2 / 4 / 8 GPUs, rounded to
# 32 as the reference's worker split does, or to the 256-wide tile).
SHARDS = [(736, 3840), (480, 3840), (3840, 3840), (480, 15360), (2944, 3840), (1920, 3840),
          (15360, 3840), (1920, 15360), (768, 3840), (512, 15360), (1472, 3840), (960, 15360)]


@pytest.mark.parametrize("nsub,K", SHARDS, ids=[f"{n}x{k}" for n, k in SHARDS])
def test_i8_resident_shard_widths_m4096(rkb, orc, nsub, K):
    import torch
    M = 4096
    A = orc.uniform_i8(300 + nsub, -128, 127, (M, K))
    B = orc.uniform_i8(400 + K, -128, 127, (nsub, K))
    ctx = rkb.lib.rocket_i8_ctx_create(1)
    assert ctx
    w = rkb.lib.rocket_i8_weights_pack(ctx, M, K, nsub, rkb.ptr(B))
    assert w
    dA = torch.from_numpy(A).cuda()
    dC = torch.full((M, nsub), -0x55555556, dtype=torch.int32, device="cuda")
    rc = rkb.lib.rocket_matmul_int8_prepacked(ctx, M, K, nsub, rkb.ptr(dA), rkb.ptr(dC), w)
    rkb.lib.rocket_i8_weights_free(ctx, w)
    rkb.lib.rocket_i8_ctx_free(ctx)
    assert rc == 0
    C = dC.cpu().numpy()
    # tile edges of the 128- and 256-row tilings, and the ends
    rows = sorted({0, 1, 127, 128, 255, 256, 511, 512, 2047, 2048, 3839, 3840, 4094, 4095})
    assert np.array_equal(C[rows], orc.matmul_int8(A[rows], B, nthreads=8))


def _ngpu():
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("nthreads", [2, 8])
def test_multi_gpu_workers_match_one(rkb, orc, nthreads):
    """Workers spread over GPUs (worker t on device t mod count): the resident
    int8 and fp16 fan-out (rocket_matmul_int8_prepacked, rocket_matmul_fp16_mt)
    with host and with device A / C is bit-identical to one worker, and the
    caller's current device is left as it was."""
    import torch
    if _ngpu() < 2 or (nthreads == 8 and _ngpu() < 8):
        pytest.skip(f"needs {min(nthreads, 8)} GPUs")
    torch.cuda.set_device(0)
    M, K, N = 256, 1024, 1024
    A = orc.uniform_i8(71, -128, 127, (M, K))
    B = orc.uniform_i8(72, -128, 127, (N, K))
    ref = orc.matmul_int8(A, B, nthreads=8)
    for nt in (1, nthreads):
        ctx = rkb.lib.rocket_i8_ctx_create(nt)
        w = rkb.lib.rocket_i8_weights_pack(ctx, M, K, N, rkb.ptr(B))
        assert ctx and w
        C = np.zeros((M, N), np.int32)
        assert rkb.lib.rocket_matmul_int8_prepacked(ctx, M, K, N, rkb.ptr(A), rkb.ptr(C), w) == 0
        assert np.array_equal(C, ref), nt
        dA = torch.from_numpy(A).cuda()
        dC = torch.zeros((M, N), dtype=torch.int32, device="cuda")
        assert rkb.lib.rocket_matmul_int8_prepacked(ctx, M, K, N, rkb.ptr(dA), rkb.ptr(dC), w) == 0
        assert torch.cuda.current_device() == 0
        assert np.array_equal(dC.cpu().numpy(), ref), nt
        rkb.lib.rocket_i8_weights_free(ctx, w)
        rkb.lib.rocket_i8_ctx_free(ctx)
    Ah = orc.normal_f16(73, 1.0 / 32, (M, K))
    Bh = orc.normal_f16(74, 1.0, (N, K))
    C1 = np.zeros((M, N), np.float16)
    Cn = np.zeros((M, N), np.float16)
    assert rkb.lib.rocket_matmul_fp16_mt(M, K, N, rkb.ptr(Ah), rkb.ptr(Bh), rkb.ptr(C1), 1) == 0
    assert rkb.lib.rocket_matmul_fp16_mt(M, K, N, rkb.ptr(Ah), rkb.ptr(Bh), rkb.ptr(Cn), nthreads) == 0
    assert np.array_equal(C1.view(np.uint16), Cn.view(np.uint16))
