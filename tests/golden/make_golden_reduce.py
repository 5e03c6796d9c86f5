"""Golden fixtures for the reduction entries, computed by the reference's OWN
host reference functions (rocket_reduce_feature_ref_fp16, rocket_cumsum_ref_fp16,
rocket_scale_rows_ref_fp16, rocket_cross_entropy_ref_fp16) built from its
sources by `make -C oracle refso` (run where the reference tree is mounted).

Inputs come from the oracle's seeded generators (reduce_golden_inputs() in
oracle/__init__.py); only outputs are stored, in reduce_golden.npz.
"""
import ctypes
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
import oracle  # noqa: E402


def P(a):
    return ctypes.c_void_p(a.ctypes.data)


def main():
    subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), "refso"], check=True, capture_output=True)
    L = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libref.so"))
    gi = oracle.reduce_golden_inputs()
    out = {}
    x = gi["x"]
    M, N = x.shape
    for mean in (0, 1):
        o = np.empty(M, np.float32)
        L.rocket_reduce_feature_ref_fp16(M, N, P(x), P(o), mean)
        out[f"red_{mean}"] = o
    for exc in (0, 1):
        for rev in (0, 1):
            y = np.empty_like(x)
            L.rocket_cumsum_ref_fp16(M, N, P(x), P(y), exc, rev)
            out[f"cum_{exc}{rev}"] = y
    y = np.empty_like(x)
    L.rocket_scale_rows_ref_fp16(M, N, P(x), P(gi["r"]), P(y))
    out["scale"] = y
    lg, t = gi["logits"], gi["target"]
    loss = np.empty(lg.shape[0], np.float32)
    L.rocket_cross_entropy_ref_fp16(lg.shape[0], lg.shape[1], P(lg), P(t), P(loss))
    out["ce"] = loss
    np.savez_compressed(os.path.join(HERE, "reduce_golden.npz"), **out)


if __name__ == "__main__":
    main()
