"""CPU: the reference's own matmul gates, compiled unchanged against the
oracle stub, pass -- the oracle is pinned to the reference's definitions.

Runs only where the reference tree is mounted (it is compiled from its own
source files); elsewhere the committed golden fixtures carry the pin.
"""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# the reference checkout: ROCKET_REF, else a directory named "reference" beside the repository
REF = os.environ.get("ROCKET_REF") or os.path.join(os.path.dirname(REPO), "reference")
ORACLE = os.path.join(REPO, "oracle")

CASES = [
    ("matmul_int8_tiled_rocket", ["64", "512", "256"]),
    ("matmul_tiled_rocket", ["64", "512", "256"]),
    ("matmul_int8_groupwise_rocket", ["32", "576", "64"]),
    ("matmul_int4_groupwise_rocket", ["16", "256", "64", "128"]),
    ("matmul_int8_prepacked_rocket", ["32", "256", "128", "2"]),
    ("matmul_int4_prepacked_rocket", ["32", "256", "128", "2"]),
    ("matmul_int4_prepacked_gw_rocket", ["32", "256", "128", "128", "2"]),
    ("matmul_mt_rocket", ["32", "256", "128"]),
]


@pytest.fixture(scope="module")
def pinned():
    if not os.path.isdir(os.path.join(REF, "tests")):
        pytest.skip("reference tree not mounted")
    subprocess.run(["make", "-C", ORACLE, "pin", f"REF={REF}"], check=True, capture_output=True)
    return os.path.join(ORACLE, "_ref")


@pytest.mark.parametrize("gate,argv", CASES, ids=[c[0] for c in CASES])
def test_reference_gate_passes_on_oracle(pinned, gate, argv):
    r = subprocess.run([os.path.join(pinned, "pin_" + gate)] + argv, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout and "FAIL" not in r.stdout, r.stdout
