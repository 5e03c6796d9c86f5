"""CPU: the oracle's reduction restatements reproduce the reference's own host
reference functions bit for bit (tests/golden/reduce_golden.npz, written by
make_golden_reduce.py from the reference's compiled sources), and the dtype
helpers keep the reference's input treatment."""
import os

import numpy as np

GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reduce_golden.npz"))


def same16(a, b):
    return np.array_equal(np.asarray(a).view(np.uint16), np.asarray(b).view(np.uint16))


def test_reduce_feature(orc):
    x = orc.reduce_golden_inputs()["x"]
    for mean in (0, 1):
        assert np.array_equal(orc.reduce_feature(x, mean), GOLD[f"red_{mean}"])


def test_cumsum_variants(orc):
    x = orc.reduce_golden_inputs()["x"]
    for exc in (0, 1):
        for rev in (0, 1):
            assert same16(orc.cumsum(x, exc, rev), GOLD[f"cum_{exc}{rev}"])


def test_scale_rows(orc):
    gi = orc.reduce_golden_inputs()
    assert same16(orc.scale_rows(gi["x"], gi["r"]), GOLD["scale"])


def test_cross_entropy_with_out_of_range_targets(orc):
    gi = orc.reduce_golden_inputs()
    loss = orc.cross_entropy(gi["logits"], gi["target"])
    assert np.array_equal(loss, GOLD["ce"])
    assert (gi["target"] < 0).any() and (gi["target"] >= gi["logits"].shape[1]).any()


def test_int16_balanced_split_matches_clamped_product(orc):
    # v = 256 hi + lo with lo = ((v + 128) & 0xFF) - 128: exact over [-32768, 32639]
    v = np.arange(-32768, 32768, dtype=np.int64)
    c = orc.int16_clamp(v)
    lo = ((c + 128) & 0xFF) - 128
    hi = (c - lo) >> 8
    assert lo.min() >= -128 and lo.max() <= 127 and hi.min() >= -128 and hi.max() <= 127
    assert np.array_equal(256 * hi + lo, c)
    assert c.max() == 32639


def test_bf16_truncation_drops_low_half(orc):
    a = np.array([1.0 + 2 ** -9, -3.14159, 1e-30], np.float32)
    t = orc.bf16_trunc(a)
    assert np.array_equal(t.view(np.uint32) & 0xFFFF, np.zeros(3, np.uint32))
    assert np.array_equal(t.view(np.uint32) >> 16, a.view(np.uint32) >> 16)
