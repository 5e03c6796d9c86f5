"""GPU: the reference's own matmul gates, compiled unchanged against
librocketnpu.so (oracle/Makefile `gates`), pass on the B200.

This is the drop-in check: the gate programs include the reference's headers,
call its API, draw its seeded inputs and apply its tolerances; only the
library underneath is ours.  The binaries are built where the reference tree
is mounted and travel with the repository (oracle/_ref is git-ignored).
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(REPO, "oracle", "_ref")

CASES = [
    ("matmul_int8_tiled_rocket", []),                       # default 128x1024x1024, srand(1234)
    ("matmul_int8_tiled_rocket", ["64", "512", "256"]),     # config 1
    ("matmul_int8_tiled_rocket", ["4096", "3840", "3840"]),
    ("matmul_tiled_rocket", []),
    ("matmul_tiled_rocket", ["512", "4096", "4096"]),       # config 2 shape
    ("matmul_int8_prepacked_rocket", []),
    ("matmul_int4_prepacked_rocket", []),
    ("matmul_mt_rocket", ["512", "3840", "4096"]),
    # widened entries: dtypes, batch, streaming, reductions
    ("matmul_bf16_tiled_rocket", ["512", "3840", "4096"]),
    ("matmul_bf16_tiled_rocket", ["1", "512", "256"]),
    ("matmul_tf32_tiled_rocket", ["512", "3840", "4096"]),
    ("matmul_tf32_tiled_rocket", ["68", "272", "144"]),
    ("matmul_int16_exact_rocket", ["256", "1024", "512"]),
    ("matmul_int16_exact_rocket", ["1", "64", "32"]),
    ("matmul_batch_rocket", []),
    ("matmul_bf16_stream_rocket", ["512", "3840", "4096", "4"]),
    ("matmul_stream_vs_prepacked_rocket", ["1024", "3840", "4096", "5", "5"]),
    ("cumsum_rocket", []),
    ("cross_entropy_rocket", []),
    ("reduce_feature_rocket", []),
    ("matmul_fp32out_rocket", ["64", "4096", "512"]),
    ("matmul_fp32out_rocket", ["1", "64", "48"]),
    ("flash_attn_rocket", []),                              # full sweep: GQA/MQA/MLA/window/softcap/long
    ("flash_attn_rocket", ["256", "1024", "128", "8", "2"]),
]


@pytest.mark.parametrize("gate,argv", CASES, ids=[f"{g}-{'x'.join(a) or 'default'}" for g, a in CASES])
def test_reference_gate_on_b200(gate, argv):
    exe = os.path.join(REF_BIN, "gate_" + gate)
    if not os.path.exists(exe):
        pytest.skip("reference gates not built (needs the reference tree at build time)")
    r = subprocess.run([exe] + argv, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "PASS" in r.stdout and "FAIL" not in r.stdout, r.stdout[-3000:]
