"""CPU: the oracle's encoder-op restatements reproduce the outputs of the
reference's own host-reference functions (tests/golden/encoder_golden.npz,
written by make_golden_encoder.py from the reference's compiled sources)."""
import os

import numpy as np
import pytest

GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "encoder_golden.npz"))


@pytest.fixture(scope="module")
def gi(orc):
    return orc.encoder_golden_inputs()


def same(a, b):
    return np.array_equal(np.asarray(a).view(np.uint16), np.asarray(b).view(np.uint16))


def test_norms(orc, gi):
    assert same(orc.layernorm(gi["ln_x"], gi["ln_g"], gi["ln_b"], 1e-5), GOLD["ln_y"])
    assert same(orc.rmsnorm(gi["ln_x"], gi["ln_g"], 1e-6), GOLD["rms_y"])


def test_softmax(orc, gi):
    assert same(orc.softmax(gi["sm_x"]), GOLD["sm_y"])
    assert same(orc.softmax(gi["sm_x"], log_mode=True), GOLD["lsm_y"])


@pytest.mark.parametrize("kind", [0, 1, 2, 3, 4, 5, 7, 8, 9, 10, 11, 12, 13, 14, 15, 18])
def test_activation(orc, gi, kind):
    src = gi["act_xp"] if kind in orc.POSITIVE_KINDS else gi["act_x"]
    assert same(orc.activation(kind, src), GOLD[f"act_y{kind}"])


def test_mha(orc, gi):
    p = gi["mha"]
    y = orc.mha_self(p["x"], p["Wq"], p["bq"], p["Wk"], p["bk"], p["Wv"], p["bv"], p["Wo"], p["bo"], 2)
    assert same(y, GOLD["mha_y"])


@pytest.mark.parametrize("kind", [3, 5])
def test_ffn(orc, gi, kind):
    y = orc.ffn(gi["ffn_x"], gi["ffn_Wg"], gi["ffn_Wu"], gi["ffn_Wd"], kind)
    assert same(y, GOLD[f"ffn_y{kind}"])


def test_encoder_block(orc, gi):
    p = gi["enc"]
    assert same(orc.encoder_block(p["x"], p, 4, 1e-5), GOLD["enc_y"])
