"""CPU: the oracle reproduces the golden fixtures made by the reference's own gates.

Each fixture in tests/golden was written by make_golden.py only after the
reference's gate (its host loop, seeded inputs and tolerance) passed on the
oracle's output; here the oracle is re-run on the stored inputs and must give
the stored outputs bit for bit (int8 / fp16) or to fp64 rounding (group-wise).
"""
import json
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MANIFEST = json.load(open(os.path.join(GOLD, "manifest.json")))


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_oracle_matches_golden(orc, name):
    meta = MANIFEST[name]
    z = np.load(os.path.join(GOLD, name + ".npz"))
    assert "PASS" in meta["gate_verdict"]
    kind = meta["kind"]
    if kind in ("int8", "int4"):
        C = orc.matmul_int8(z["A"], z["B"])
        assert np.array_equal(C, z["C"])
    elif kind == "fp16":
        _, C16 = orc.matmul_fp16(z["A"], z["B"])
        assert np.array_equal(C16.view(np.uint16), z["C"].view(np.uint16))
    else:
        ref = orc.gw_ref(z["A"], z["B"], z["a_scale"], z["b_scale"], meta["group"])
        np.testing.assert_allclose(ref.astype(np.float32), z["C"], rtol=0, atol=0)


def test_oracle_int8_matches_numpy(orc):
    A = orc.uniform_i8(1, -128, 127, (37, 96))
    B = orc.uniform_i8(2, -128, 127, (40, 96))
    ref = (A.astype(np.int64) @ B.astype(np.int64).T).astype(np.int32)
    assert np.array_equal(orc.matmul_int8(A, B, nthreads=3), ref)


def test_oracle_gw_f32_close_to_fp64(orc):
    A = orc.uniform_i8(3, -127, 127, (8, 256))
    B = orc.uniform_i8(4, -8, 7, (16, 256))
    a = orc.uniform_f32(5, 0.5, 1.5, (8, 8))
    b = orc.uniform_f32(6, 0.5, 1.5, (16, 8))
    r64 = orc.gw_ref(A, B, a, b, 32)
    r32 = orc.gw_f32(A, B, a, b, 32)
    rms = np.sqrt(np.mean(r64 ** 2))
    assert np.max(np.abs(r32 - r64)) <= 1e-5 * rms


def test_generators_deterministic(orc):
    assert np.array_equal(orc.uniform_i8(7, -8, 7, 100), orc.uniform_i8(7, -8, 7, 100))
    x = orc.uniform_i8(7, -8, 7, 100000)
    assert x.min() == -8 and x.max() == 7
    n = orc.normal_f16(9, 1.0, 200000).astype(np.float64)
    assert abs(n.mean()) < 0.01 and abs(n.std() - 1) < 0.01
    g = orc.glibc_i8(1234, -128, 256, 4)
    # glibc rand() after srand(1234): the stream the reference's int8 gate draws
    assert g.dtype == np.int8 and len(g) == 4
