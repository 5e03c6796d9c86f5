"""CPU: the oracle's masked grouped-query attention reproduces the reference's own
host reference (rocket_flash_attn_ref_fp16) bit for bit on the golden cases
(tests/golden/fa_golden.npz, written by make_golden_fa.py): GQA and MQA head
maps, sliding window, soft-cap, MLA (dh != dv), ragged T / n_kv."""
import os

import numpy as np
import pytest

GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fa_golden.npz"))


@pytest.mark.parametrize("i", range(5))
def test_flash_attn_golden(orc, i):
    case = orc.FA_GOLDEN_CASES[i]
    Q, K, V, M = orc.fa_golden_inputs(case)
    y = orc.flash_attn(Q, K, V, M, float(np.float32(1.0 / np.sqrt(case[2]))), case[7])
    assert np.array_equal(y.view(np.uint16), GOLD[f"fa{i}"].view(np.uint16))


def test_fully_masked_row_averages_values(orc):
    # every key masked: scores clamp to -30000, so the row is the mean of V
    Q = orc.normal_f16(5, 1.0, (1, 4, 32))
    K = orc.normal_f16(6, 1.0, (1, 8, 32))
    V = orc.normal_f16(7, 1.0, (1, 32, 8))
    M = np.full((4, 8), -np.inf, np.float16)
    y = orc.flash_attn(Q, K, V, M, 0.1)
    np.testing.assert_allclose(y[0].astype(np.float64), np.broadcast_to(V[0].astype(np.float64).mean(1), (4, 32)),
                               atol=1e-3)
