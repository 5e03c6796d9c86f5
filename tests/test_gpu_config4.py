"""GPU parity at BASELINE config 4's own shape: transformer encoder block,
fp16, d_model 512, 8 heads (head_dim 64), d_ff 2048, T = 1500, batch 4;
activations N(0,1), weights N(0,0.02), LayerNorm gamma 1 / beta 0.

Both forms are checked against the oracle (the reference's
rocket_encoder_block_ref_fp16, restated and pinned bit-for-bit to the
reference's own function) under the reference gate's bound
(tests/encoder_block_rocket.c:66-71: cosine >= 0.9995 and
max_abs <= 0.03 * max|ref| + 2e-3) and the north-star fp16 bound:
  - rocket_encoder_block_fp16 once per sequence (the reference API);
  - rocket_b200_encoder_block_batched_fp16 over the stacked batch (the form
    the bench times).
"""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

T, D, NH, DFF, NB = 1500, 512, 8, 2048, 4


def check(orc, got, ref):
    g = np.asarray(got, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    assert np.isfinite(g).all()
    fro, mar = orc.rel_frobenius(g, r), orc.max_abs_rel(g, r)
    cos = float(g @ r / (np.linalg.norm(g) * np.linalg.norm(r) + 1e-300))
    assert fro <= 1e-2 and mar <= 2e-2, (fro, mar)
    assert cos >= 0.9995 and np.max(np.abs(g - r)) <= 0.03 * np.max(np.abs(r)) + 2e-3, cos


@pytest.fixture(scope="module")
def batch(orc):
    p = orc.encoder_params(T, D, NH, DFF, 4000)
    xs = [orc.normal_f16(4100 + b, 1.0, (T, D)) for b in range(NB)]
    with ThreadPoolExecutor(NB) as ex:
        refs = list(ex.map(lambda x: orc.encoder_block(x, p, NH, 1e-5), xs))
    return p, xs, refs


def test_config4_per_sequence(rkb, dev, orc, batch):
    p, xs, refs = batch
    for x, ref in zip(xs, refs):
        y = np.zeros((T, D), np.float16)
        assert rkb.lib.rocket_encoder_block_fp16(dev.fd, T, D, NH, DFF, rkb.ptr(x),
                                                 *[rkb.ptr(p[k]) for k in rkb.ENCODER_KEYS], 1e-5,
                                                 rkb.ptr(y)) == 0
        check(orc, y, ref)


def test_config4_batched(rkb, dev, orc, batch):
    p, xs, refs = batch
    x = np.ascontiguousarray(np.concatenate(xs, axis=0))
    y = np.zeros((NB * T, D), np.float16)
    assert rkb.lib.rocket_b200_encoder_block_batched_fp16(dev.fd, NB, T, D, NH, DFF, rkb.ptr(x),
                                                          *[rkb.ptr(p[k]) for k in rkb.ENCODER_KEYS],
                                                          1e-5, rkb.ptr(y)) == 0
    for b in range(NB):
        check(orc, y[b * T:(b + 1) * T], refs[b])
