"""Golden outputs for masked grouped-query attention, computed by the reference's
OWN host reference rocket_flash_attn_ref_fp16 (src/rocket_attn.c:189-222), built
from its sources by `make -C oracle refso` (run where the reference tree is
mounted).  Inputs come from oracle.fa_golden_inputs(case) for each case of
oracle.FA_GOLDEN_CASES; only outputs are stored, in fa_golden.npz."""
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
    L.rocket_flash_attn_ref_fp16.argtypes = [ctypes.c_int] * 6 + [ctypes.c_float] * 2 + [ctypes.c_void_p] * 5
    out = {}
    for i, case in enumerate(oracle.FA_GOLDEN_CASES):
        T, n_kv, dh, dv, nh, nkvh, _, cap = case
        Q, K, V, M = oracle.fa_golden_inputs(case)
        o = np.empty((nh, T, dv), np.float16)
        L.rocket_flash_attn_ref_fp16(T, n_kv, dh, dv, nh, nkvh, 1.0 / np.sqrt(dh), cap, P(Q), P(K), P(V),
                                     P(M), P(o))
        out[f"fa{i}"] = o
    np.savez_compressed(os.path.join(HERE, "fa_golden.npz"), **out)


if __name__ == "__main__":
    main()
