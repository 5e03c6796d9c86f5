"""GPU: the reference's own matmul gates, compiled unchanged against
librocketnpu.so (oracle/Makefile `gates`), pass on the B200.

This is the drop-in check: the gate programs include the reference's headers,
call its API, draw its seeded inputs and apply its tolerances; only the
library underneath is ours.  The binaries are built where the reference tree
is mounted and travel with the repository (oracle/_ref is git-ignored).
"""
import os
import re
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
    # group-wise: the reference's 1e-5 * rms bound against fp64, resident == one-shot
    ("matmul_int8_groupwise_rocket", []),                   # groups 96 .. 2880
    ("matmul_int4_groupwise_rocket", []),
    ("matmul_int4_groupwise_rocket", ["2048", "3840", "1024", "32"]),
    ("matmul_int4_prepacked_gw_rocket", []),
    ("matmul_int8_prepacked_gw_rocket", []),
    ("matmul_int8_prepacked_gw_rocket", ["256", "2880", "512", "1440"]),
    ("matmul_int8_crossm_gw_rocket", []),
    # resident weights across M, cross-M reuse, other dtypes' one-shot gates
    ("matmul_prepacked_rocket", []),
    ("matmul_prepacked_crossm_rocket", []),
    ("matmul_int8_crossm_rocket", []),
    ("matmul_int4_crossm_rocket", []),
    ("matmul_int4_tiled_rocket", []),
    # encoder ops and block (their checkers are the reference's *_ref_fp16)
    ("encoder_block_rocket", []),
    ("layernorm_rocket", []),
    ("rmsnorm_rocket", []),
    ("softmax_rocket", []),
    ("mha_rocket", []),
    ("ffn_rocket", []),
    ("ffn_fused_rocket", []),
    ("gelu_rocket", []),
    ("ew_minmax_rocket", []),
]

# The reference's correctness matrix (tests/correctness_matrix.sh:52-131):
# cosine >= 0.9995 on sampled rows, exact for the integer dtypes.
SHAPES = [(3840, 4096), (3840, 2048), (4096, 3840), (3840, 15360), (15360, 3840), (1024, 1024),
          (8224, 2048), (3840, 4112)]
MATRIX = []
for K, N in SHAPES:                                                   # part 1: fp16 shape grid
    for M in (1, 4, 130, 256, 300, 512):
        MATRIX.append(((str(M), str(K), str(N), "tiled"), "48"))
for K, N in ((3840, 4096), (15360, 3840)):                           # part 2: entry points
    for mode in ("tiled", "mt", "stream", "prepacked"):
        for M in (1, 4, 512):
            MATRIX.append(((str(M), str(K), str(N), mode), "48"))
for dt in ("int8", "int4", "int16", "bf16", "tf32"):                  # part 4: dtype matrix
    for K, N in ((3840, 4096), (3840, 2048), (3840, 15360), (15360, 3840)):
        for M in (1, 4, 512):
            MATRIX.append(((str(M), str(K), str(N), "tiled", dt), "32"))
for dt in ("int8", "int4"):                                           # part 5: resident
    for M in (1, 4, 512):
        MATRIX.append(((str(M), "3840", "4096", "prepacked", dt), "32"))


@pytest.mark.parametrize("gate,argv", CASES, ids=[f"{g}-{'x'.join(a) or 'default'}" for g, a in CASES])
def test_reference_gate_on_b200(gate, argv):
    exe = os.path.join(REF_BIN, "gate_" + gate)
    if not os.path.exists(exe):
        pytest.skip("reference gates not built (needs the reference tree at build time)")
    r = subprocess.run([exe] + argv, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "PASS" in r.stdout and not failed_lines(r.stdout), r.stdout[-3000:]


def failed_lines(out):
    """Lines of a gate's output that report a failure ("0/3 FAILED" is a count, not one)."""
    return [ln for ln in out.splitlines() if "FAIL" in ln and not re.search(r"\b0/\d+ FAILED", ln)]


@pytest.mark.parametrize("argv,rows", MATRIX, ids=["-".join(a) for a, _ in MATRIX])
def test_correctness_matrix_on_b200(argv, rows):
    exe = os.path.join(REF_BIN, "gate_matmul_correctness_matrix_rocket")
    if not os.path.exists(exe):
        pytest.skip("reference gates not built (needs the reference tree at build time)")
    env = dict(os.environ, SAMPLE_ROWS=rows)
    r = subprocess.run([exe] + list(argv), capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    # SKIP is the reference's verdict when a path declines a shape; only resident
    # weights at M == 1 may do that (correctness_matrix.sh part 5), all else must PASS
    may_skip = argv[3] == "prepacked" and argv[0] == "1"
    ok = "PASS" in r.stdout or (may_skip and "SKIP" in r.stdout)
    assert ok and "FAIL" not in r.stdout, r.stdout[-3000:]
