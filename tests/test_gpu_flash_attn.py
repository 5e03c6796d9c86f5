"""GPU parity of masked grouped-query attention (rocket_flash_attn_fp16 / _mt /
_ctx) through the C ABI against the oracle and the golden outputs of the
reference's own host reference.

Bar: the reference gate's (tests/flash_attn_rocket.c:96-103): cosine >= 0.9995
and max|got-ref| <= 0.02 max|ref| + 1e-3; plus relative Frobenius <= 5e-3.  P is
rounded to fp16 before P.V (as in any fp16 attention), which bounds the error.
"""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fa_golden.npz"))


def P(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def check(got, ref):
    g = got.astype(np.float64).ravel()
    r = ref.astype(np.float64).ravel()
    assert np.isfinite(g).all()
    cos = g @ r / (np.linalg.norm(g) * np.linalg.norm(r) + 1e-30)
    mx = np.max(np.abs(g - r))
    fro = np.linalg.norm(g - r) / (np.linalg.norm(r) + 1e-30)
    assert cos >= 0.9995 and mx <= 0.02 * np.max(np.abs(r)) + 1e-3 and fro <= 5e-3, (cos, mx, fro)


def run(rkb, fd, Q, K, V, M, scale, cap, entry="single", ctx=None):
    nh, T, dh = Q.shape
    nkvh, n_kv, _ = K.shape
    dv = V.shape[1]
    out = np.full((nh, T, dv), np.nan, np.float16)
    args = (T, n_kv, dh, dv, nh, nkvh, scale, cap, P(Q), P(K), P(V), P(M), P(out))
    if entry == "single":
        rc = rkb.lib.rocket_flash_attn_fp16(fd, *args)
    elif entry == "mt":
        rc = rkb.lib.rocket_flash_attn_fp16_mt(fd, *args, 5)
    else:
        rc = rkb.lib.rocket_flash_attn_fp16_ctx(ctx, *args)
    assert rc == 0
    return out


@pytest.mark.parametrize("i", range(5))
def test_golden(rkb, dev, orc, i):
    case = orc.FA_GOLDEN_CASES[i]
    Q, K, V, M = orc.fa_golden_inputs(case)
    out = run(rkb, dev.fd, Q, K, V, M, float(1.0 / np.sqrt(case[2])), case[7])
    check(out, GOLD[f"fa{i}"])


# (T, n_kv, dh, dv, nh, nkvh, window, softcap, masked)
CASES = [
    (128, 128, 256, 256, 4, 2, 0, 0.0, True),     # Gemma-style local layer, GQA 2:1
    (128, 128, 256, 256, 4, 1, 64, 0.0, True),    # MQA + sliding window
    (100, 100, 256, 256, 2, 1, 0, 0.0, True),     # T % 4, n_kv % 32 (ragged V pitch)
    (64, 512, 128, 128, 4, 2, 0, 0.0, True),      # cached prefix (n_kv > T), BKV 128
    (128, 128, 64, 64, 4, 4, 0, 50.0, True),      # soft-cap
    (128, 128, 192, 128, 4, 1, 0, 0.0, True),     # MLA: dh 192, dv 128
    (200, 333, 96, 48, 3, 3, 0, 0.0, False),      # no mask; dh 96 (zero-filled panel), dv 48
    (300, 300, 32, 16, 2, 1, 17, 0.0, True),      # tiny heads, odd window
    (64, 4096, 256, 256, 2, 1, 0, 0.0, True),     # long context (64 key blocks)
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "T{}kv{}dh{}dv{}h{}/{}w{}c{}m{}".format(*c))
def test_vs_oracle(rkb, dev, orc, case):
    T, n_kv, dh, dv, nh, nkvh, window, cap, masked = case
    seed = T + n_kv + dh
    Q = orc.normal_f16(seed + 1, 1.0, (nh, T, dh))
    K = orc.normal_f16(seed + 2, 1.0, (nkvh, n_kv, dh))
    V = orc.normal_f16(seed + 3, 1.0, (nkvh, dv, n_kv))
    M = orc.causal_mask(T, n_kv, window) if masked else None
    scale = float(1.0 / np.sqrt(dh))
    ref = orc.flash_attn(Q, K, V, M, scale, cap)
    check(run(rkb, dev.fd, Q, K, V, M, scale, cap), ref)


def test_fully_masked_rows_and_entries_agree(rkb, dev, orc):
    T, n_kv, dh, nh = 64, 96, 64, 2
    Q = orc.normal_f16(1, 1.0, (nh, T, dh))
    K = orc.normal_f16(2, 1.0, (1, n_kv, dh))
    V = orc.normal_f16(3, 1.0, (1, dh, n_kv))
    M = orc.causal_mask(T, n_kv)
    M[:5] = -np.inf                                   # rows with every key masked
    scale = 0.125
    ref = orc.flash_attn(Q, K, V, M, scale)
    a = run(rkb, dev.fd, Q, K, V, M, scale, 0.0)
    check(a, ref)
    b = run(rkb, dev.fd, Q, K, V, M, scale, 0.0, entry="mt")
    ctx = rkb.lib.rocket_fa_ctx_create(5)
    assert ctx
    try:
        c1 = run(rkb, dev.fd, Q, K, V, M, scale, 0.0, entry="ctx", ctx=ctx)
        c2 = run(rkb, dev.fd, Q, K, V, M, scale, 0.0, entry="ctx", ctx=ctx)
    finally:
        rkb.lib.rocket_fa_ctx_free(ctx)
    for x in (b, c1, c2):
        assert np.array_equal(x.view(np.uint16), a.view(np.uint16))


def test_rejects_bad_shapes(rkb, dev, orc):
    Q = np.zeros((3, 8, 64), np.float16)
    K = np.zeros((2, 8, 64), np.float16)
    V = np.zeros((2, 64, 8), np.float16)
    out = np.zeros((3, 8, 64), np.float16)
    # n_head % n_kv_heads != 0
    assert rkb.lib.rocket_flash_attn_fp16(dev.fd, 8, 8, 64, 64, 3, 2, 0.1, 0.0, P(Q), P(K), P(V), None, P(out)) != 0
    # head_dim above what the kernel takes
    assert rkb.lib.rocket_flash_attn_fp16(dev.fd, 8, 8, 320, 64, 2, 2, 0.1, 0.0, P(Q), P(K), P(V), None, P(out)) != 0
