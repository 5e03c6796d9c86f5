"""GPU parity for the encoder ops against the oracle (pinned bit-for-bit to
the reference's own host references) and against the reference-generated
golden outputs.  Tolerances: the north-star fp16 bound (relative Frobenius
<= 1e-2, max-abs relative <= 2e-2) plus the reference's encoder gate
(tests/encoder_block_rocket.c:66-71: cosine >= 0.9995 and
max_abs <= 0.03 * max|ref| + 2e-3)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "encoder_golden.npz"))


def check(orc, got, ref, fro_tol=1e-2, mar_tol=2e-2):
    g = np.asarray(got, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    assert np.isfinite(g).all()
    fro, mar = orc.rel_frobenius(g, r), orc.max_abs_rel(g, r)
    cos = float(g @ r / (np.linalg.norm(g) * np.linalg.norm(r) + 1e-300))
    assert fro <= fro_tol and mar <= mar_tol, (fro, mar)
    assert cos >= 0.9995 and np.max(np.abs(g - r)) <= 0.03 * np.max(np.abs(r)) + 2e-3, cos
    return fro


@pytest.fixture(scope="module")
def gi(orc):
    return orc.encoder_golden_inputs()


def P(rkb, a):
    return rkb.ptr(a)


def test_layernorm_rmsnorm(rkb, dev, orc, gi):
    x, g, b = gi["ln_x"], gi["ln_g"], gi["ln_b"]
    y = np.zeros_like(x)
    assert rkb.lib.rocket_layernorm_fp16(dev.fd, 37, 512, P(rkb, x), P(rkb, g), P(rkb, b), 1e-5, P(rkb, y)) == 0
    assert check(orc, y, GOLD["ln_y"]) < 2e-3
    assert rkb.lib.rocket_rmsnorm_fp16(dev.fd, 37, 512, P(rkb, x), P(rkb, g), 1e-6, P(rkb, y)) == 0
    assert check(orc, y, GOLD["rms_y"]) < 2e-3


@pytest.mark.parametrize("M,H", [(1, 64), (6000, 512), (5, 100), (3, 4096)])
def test_layernorm_shapes(rkb, dev, orc, M, H):
    x = orc.normal_f16(M + H, 1.5, (M, H))
    g = orc.normal_f16(7, 1.0, (H,))
    b = orc.normal_f16(8, 0.3, (H,))
    y = np.zeros_like(x)
    assert rkb.lib.rocket_layernorm_fp16(dev.fd, M, H, P(rkb, x), P(rkb, g), P(rkb, b), 1e-5, P(rkb, y)) == 0
    check(orc, y, orc.layernorm(x, g, b, 1e-5))


def test_softmax(rkb, dev, orc, gi):
    x = gi["sm_x"]
    y = np.zeros_like(x)
    assert rkb.lib.rocket_softmax_fp16(dev.fd, 21, 1500, P(rkb, x), P(rkb, y)) == 0
    check(orc, y, GOLD["sm_y"])
    assert np.allclose(y.astype(np.float32).sum(1), 1.0, atol=5e-3)
    assert rkb.lib.rocket_logsoftmax_fp16(dev.fd, 21, 1500, P(rkb, x), P(rkb, y)) == 0
    check(orc, y, GOLD["lsm_y"])


@pytest.mark.parametrize("kind", [0, 1, 2, 3, 4, 5, 7, 8, 9, 10, 11, 12, 13, 14, 15, 18])
def test_activation(rkb, dev, orc, gi, kind):
    src = gi["act_xp"] if kind in orc.POSITIVE_KINDS else gi["act_x"]
    y = np.zeros_like(src)
    assert rkb.lib.rocket_activation_fp16(dev.fd, kind, P(rkb, src), P(rkb, y), src.size) == 0
    r = GOLD[f"act_y{kind}"].astype(np.float64)
    # element-wise: every value within 2 fp16 ulps of the fp64 result
    assert np.all(np.abs(y.astype(np.float64) - r) <= 2 * np.spacing(np.abs(r).astype(np.float16)).astype(np.float64) + 1e-7)


def test_activation_parametric_kinds_refused(rkb, dev):
    x = np.zeros(64, np.float16)
    for k in (6, 16, 17):
        assert rkb.lib.rocket_activation_fp16(dev.fd, k, P(rkb, x), P(rkb, x), 64) == rkb.ROCKET_E_UNSUPPORTED


def test_elementwise_binary(rkb, dev, orc):
    n = 10007   # odd length: vector body + scalar tail
    a = orc.normal_f16(1, 1.0, (n,))
    b = orc.normal_f16(2, 1.0, (n,))
    y = np.zeros_like(a)
    for fn, ref in [(rkb.lib.rocket_ew_add_fp16, a.astype(np.float32) + b), (rkb.lib.rocket_ew_mul_fp16, a.astype(np.float32) * b),
                    (rkb.lib.rocket_ew_sub_fp16, a.astype(np.float32) - b)]:
        assert fn(dev.fd, P(rkb, a), P(rkb, b), P(rkb, y), n) == 0
        assert np.array_equal(y, ref.astype(np.float16))


@pytest.mark.parametrize("kind", [3, 5])
def test_ffn(rkb, dev, orc, gi, kind):
    y = np.zeros((16, 128), np.float16)
    assert rkb.lib.rocket_ffn_fp16(dev.fd, 16, 128, 256, P(rkb, gi["ffn_x"]), P(rkb, gi["ffn_Wg"]), P(rkb, gi["ffn_Wu"]),
                                   P(rkb, gi["ffn_Wd"]), kind, P(rkb, y)) == 0
    check(orc, y, GOLD[f"ffn_y{kind}"])


def test_mlp_fused(rkb, dev, orc):
    M, Din, Dff, Dout = 100, 256, 1024, 256
    x = orc.normal_f16(1, 1.0, (M, Din))
    W1 = orc.normal_f16(2, 0.05, (Dff, Din))
    b1 = orc.normal_f16(3, 0.05, (Dff,))
    W2 = orc.normal_f16(4, 0.05, (Dout, Dff))
    y = np.zeros((M, Dout), np.float16)
    assert rkb.lib.rocket_mlp_fp16_fused(dev.fd, M, Din, Dff, Dout, P(rkb, x), P(rkb, W1), P(rkb, b1), P(rkb, W2),
                                         5, P(rkb, y)) == 0
    h = x.astype(np.float64) @ W1.astype(np.float64).T + b1
    from math import erf, sqrt
    g = 0.5 * h * (1 + np.vectorize(erf)(h / sqrt(2)))
    check(orc, y, g @ W2.astype(np.float64).T)


def test_mha_golden(rkb, dev, orc, gi):
    p = gi["mha"]
    y = np.zeros((40, 128), np.float16)
    args = [P(rkb, p[k]) for k in ["x", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo"]]
    assert rkb.lib.rocket_mha_self_fp16(dev.fd, 40, 128, 2, *args, P(rkb, y)) == 0
    check(orc, y, GOLD["mha_y"])


@pytest.mark.parametrize("T,d,nh", [(1, 64, 1), (128, 128, 2), (129, 256, 4), (300, 512, 8)])
def test_mha_shapes(rkb, dev, orc, T, d, nh):
    p = orc.encoder_params(T, d, nh, 4 * d, T + d)
    y = np.zeros((T, d), np.float16)
    args = [P(rkb, p[k]) for k in ["x", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo"]]
    assert rkb.lib.rocket_mha_self_fp16(dev.fd, T, d, nh, *args, P(rkb, y)) == 0
    ref = orc.mha_self(p["x"], p["Wq"], p["bq"], p["Wk"], p["bk"], p["Wv"], p["bv"], p["Wo"], p["bo"], nh)
    check(orc, y, ref)


@pytest.mark.parametrize("T,d,nh", [(16, 128, 4),      # head_dim 32
                                    (200, 512, 4),     # head_dim 128
                                    (77, 512, 2)])     # head_dim 256
def test_mha_other_head_dims(rkb, dev, orc, T, d, nh):
    """head_dim != 64 runs the flash kernel over the split heads.  Wq / Wk are
    drawn large enough that the softmax is far from uniform."""
    p = orc.encoder_params(T, d, nh, 4 * d, T + d + 1)
    p["Wq"] = orc.normal_f16(T + 901, 2.0 / np.sqrt(d), (d, d))
    p["Wk"] = orc.normal_f16(T + 902, 2.0 / np.sqrt(d), (d, d))
    y = np.zeros((T, d), np.float16)
    args = [P(rkb, p[k]) for k in ["x", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo"]]
    assert rkb.lib.rocket_mha_self_fp16(dev.fd, T, d, nh, *args, P(rkb, y)) == 0
    ref = orc.mha_self(p["x"], p["Wq"], p["bq"], p["Wk"], p["bk"], p["Wv"], p["bv"], p["Wo"], p["bo"], nh)
    check(orc, y, ref)


def test_mha_unsupported_head_dim(rkb, dev, orc):
    p = orc.encoder_params(16, 160, 4, 320, 1)   # head_dim 40: not a multiple of 16
    y = np.zeros((16, 160), np.float16)
    args = [P(rkb, p[k]) for k in ["x", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo"]]
    assert rkb.lib.rocket_mha_self_fp16(dev.fd, 16, 160, 4, *args, P(rkb, y)) == rkb.ROCKET_E_UNSUPPORTED


def test_encoder_block_head_dim_128(rkb, dev, orc):
    T, d, nh, dff = 96, 512, 4, 1024
    p = orc.encoder_params(T, d, nh, dff, 11)
    y = np.zeros((T, d), np.float16)
    assert rkb.lib.rocket_encoder_block_fp16(dev.fd, T, d, nh, dff, P(rkb, p["x"]),
                                             *[P(rkb, p[k]) for k in rkb.ENCODER_KEYS], 1e-5, P(rkb, y)) == 0
    check(orc, y, orc.encoder_block(p["x"], p, nh, 1e-5))


def test_encoder_block_golden(rkb, dev, orc, gi):
    p = gi["enc"]
    y = np.zeros((64, 256), np.float16)
    assert rkb.lib.rocket_encoder_block_fp16(dev.fd, 64, 256, 4, 1024, P(rkb, p["x"]),
                                             *[P(rkb, p[k]) for k in rkb.ENCODER_KEYS], 1e-5, P(rkb, y)) == 0
    check(orc, y, GOLD["enc_y"])


@pytest.mark.parametrize("T,d,nh,dff", [(100, 512, 8, 2048), (257, 512, 8, 2048)])
def test_encoder_block_vs_oracle(rkb, dev, orc, T, d, nh, dff):
    p = orc.encoder_params(T, d, nh, dff, 7 + T)
    y = np.zeros((T, d), np.float16)
    assert rkb.lib.rocket_encoder_block_fp16(dev.fd, T, d, nh, dff, P(rkb, p["x"]),
                                             *[P(rkb, p[k]) for k in rkb.ENCODER_KEYS], 1e-5, P(rkb, y)) == 0
    check(orc, y, orc.encoder_block(p["x"], p, nh, 1e-5))


def test_encoder_batched_equals_per_sequence(rkb, dev, orc):
    """Config 4 layout (d=512, 8 heads, d_ff=2048) at T=300, nb=3: the batched
    extension equals three single-sequence calls bit for bit (same kernels, same
    per-row arithmetic), and each matches the oracle."""
    import torch
    T, d, nh, dff, nb = 300, 512, 8, 2048, 3
    p = orc.encoder_params(T, d, nh, dff, 99)
    xs = np.concatenate([orc.normal_f16(500 + i, 1.0, (T, d)) for i in range(nb)])
    dp = {k: torch.from_numpy(p[k]).cuda() for k in rkb.ENCODER_KEYS}
    dx = torch.from_numpy(xs).cuda()
    dy = torch.zeros_like(dx)
    assert rkb.lib.rocket_b200_encoder_block_batched_fp16(dev.fd, nb, T, d, nh, dff, P(rkb, dx),
                                                          *[P(rkb, dp[k]) for k in rkb.ENCODER_KEYS], 1e-5,
                                                          P(rkb, dy)) == 0
    yb = dy.cpu().numpy()
    for i in range(nb):
        yi = np.zeros((T, d), np.float16)
        assert rkb.lib.rocket_encoder_block_fp16(dev.fd, T, d, nh, dff, P(rkb, xs[i * T:(i + 1) * T].copy()),
                                                 *[P(rkb, p[k]) for k in rkb.ENCODER_KEYS], 1e-5, P(rkb, yi)) == 0
        assert np.array_equal(yi.view(np.uint16), yb[i * T:(i + 1) * T].view(np.uint16))
        if i == 0:
            check(orc, yi, orc.encoder_block(xs[:T], p, nh, 1e-5))


def test_async_enqueue_with_device_operands(rkb, dev, orc, gi):
    """rocket_b200_set_async: with device inputs and outputs the encoder entries
    return after the launches; rocket_b200_sync collects the status."""
    import torch
    x, g, b = (torch.from_numpy(gi[k]).cuda() for k in ("ln_x", "ln_g", "ln_b"))
    y = torch.zeros_like(x)
    p = gi["enc"]
    T, d = p["x"].shape
    pe = {k: torch.from_numpy(np.ascontiguousarray(p[k])).cuda() for k in ["x"] + list(rkb.ENCODER_KEYS)}
    ye = torch.zeros((T, d), dtype=torch.float16, device="cuda")
    rkb.lib.rocket_b200_set_async(1)
    try:
        for _ in range(3):
            assert rkb.lib.rocket_layernorm_fp16(dev.fd, x.shape[0], x.shape[1], x.data_ptr(), g.data_ptr(),
                                                 b.data_ptr(), 1e-5, y.data_ptr()) == 0
            assert rkb.lib.rocket_encoder_block_fp16(dev.fd, T, d, 4, 1024, pe["x"].data_ptr(),
                                                     *[pe[k].data_ptr() for k in rkb.ENCODER_KEYS], 1e-5,
                                                     ye.data_ptr()) == 0
        assert rkb.lib.rocket_b200_sync(dev.fd) == 0
    finally:
        rkb.lib.rocket_b200_set_async(0)
    check(orc, y.cpu().numpy(), GOLD["ln_y"])
    check(orc, ye.cpu().numpy(), GOLD["enc_y"])


def test_mha_lazy_rescale(rkb, dev, orc):
    """Scores that jump by far more than 2^8 (log2 units) in later key blocks,
    so the head_dim-64 kernel's in-TMEM rescale of O (lazy rescaling) runs,
    twice per row for the rows that see both jumps, with P double-buffered."""
    T, d, nh = 384, 64, 1
    p = orc.encoder_params(T, d, nh, 4 * d, 77)
    x = orc.normal_f16(78, 0.3, (T, d)).astype(np.float32)
    v = np.ones(T, np.float32)
    v[[130, 131, 200]] = 3.0          # key block 1: raw score x5 per unit -> jump of ~10
    v[[300, 301]] = 6.0               # key block 2: a second, larger jump
    x[:, 0] = v
    p["x"] = x.astype(np.float16)
    Wq = orc.normal_f16(79, 0.02, (d, d)).astype(np.float32)
    Wk = orc.normal_f16(80, 0.02, (d, d)).astype(np.float32)
    Wq[0, :] = 0.0
    Wk[0, :] = 0.0
    Wq[0, 0] = 40.0                   # q_t[0] = 40 v_t, k_s[0] = v_s: scaled score 5 v_t v_s
    Wk[0, 0] = 1.0
    p["Wq"], p["Wk"] = Wq.astype(np.float16), Wk.astype(np.float16)
    p["bq"] = np.zeros(d, np.float16)
    p["bk"] = np.zeros(d, np.float16)
    p["Wv"] = orc.normal_f16(81, 0.5, (d, d))
    y = np.zeros((T, d), np.float16)
    args = [P(rkb, p[k]) for k in ["x", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo"]]
    assert rkb.lib.rocket_mha_self_fp16(dev.fd, T, d, nh, *args, P(rkb, y)) == 0
    ref = orc.mha_self(p["x"], p["Wq"], p["bq"], p["Wk"], p["bk"], p["Wv"], p["bv"], p["Wo"], p["bo"], nh)
    check(orc, y, ref)


@pytest.mark.parametrize("n", [1, 8, 1003, 1 << 20])
def test_ew_max_min_clip(rkb, dev, orc, n):
    a = orc.normal_f16(n + 1, 2.0, (n,))
    b = orc.normal_f16(n + 2, 2.0, (n,))
    y = np.zeros(n, np.float16)
    assert rkb.lib.rocket_ew_max_fp16(dev.fd, P(rkb, a), P(rkb, b), P(rkb, y), n) == 0
    assert np.array_equal(y, np.maximum(a, b))
    assert rkb.lib.rocket_ew_min_fp16(dev.fd, P(rkb, a), P(rkb, b), P(rkb, y), n) == 0
    assert np.array_equal(y, np.minimum(a, b))
    assert rkb.lib.rocket_clip_fp16(dev.fd, -1.0, 0.5, P(rkb, a), P(rkb, y), n) == 0
    assert np.array_equal(y, np.clip(a, np.float16(-1.0), np.float16(0.5)))
    assert rkb.lib.rocket_clip_fp16(dev.fd, 1.0, -1.0, P(rkb, a), P(rkb, y), n) == rkb.ROCKET_E_SHAPE
    assert rkb.lib.rocket_activation_name(5) == b"gelu" and rkb.lib.rocket_activation_name(99) == b"?"
