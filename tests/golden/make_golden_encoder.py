"""Golden fixtures for the encoder ops, computed by the reference's OWN host
reference functions (rocket_layernorm_ref_fp16, rocket_rmsnorm_ref_fp16,
rocket_softmax_ref_fp16, rocket_logsoftmax_ref_fp16, rocket_activation_ref_fp16,
rocket_mha_self_ref_fp16, rocket_ffn_ref_fp16, rocket_encoder_block_ref_fp16),
built from the reference's sources by `make -C oracle refso` (needs the
reference tree, so run it in the container where it is mounted).

Inputs are seeded (oracle generators); shapes follow the reference's gates
(tests/encoder_block_rocket.c:90-92 uses (T,d,heads,dff) = (64,256,4,1024)).
Only the outputs are stored (encoder_golden.npz next to this script); the
inputs are regenerated from the same seeds by the oracle's generators (see
golden_inputs() in tests/test_gpu_encoder.py and oracle.encoder_params).
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


def ref_lib():
    subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), "refso"], check=True, capture_output=True)
    return ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libref.so"))


def P(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def main():
    L = ref_lib()
    F = ctypes.c_float
    out = {}
    gi = oracle.encoder_golden_inputs()
    # layernorm / rmsnorm
    x, g, b = gi["ln_x"], gi["ln_g"], gi["ln_b"]
    y = np.empty_like(x)
    L.rocket_layernorm_ref_fp16(37, 512, P(x), P(g), P(b), F(1e-5), P(y))
    out.update(ln_y=y.copy())
    L.rocket_rmsnorm_ref_fp16(37, 512, P(x), P(g), F(1e-6), P(y))
    out.update(rms_y=y.copy())
    # softmax / logsoftmax
    s = gi["sm_x"]
    ys = np.empty_like(s)
    L.rocket_softmax_ref_fp16(21, 1500, P(s), P(ys))
    out.update(sm_y=ys.copy())
    L.rocket_logsoftmax_ref_fp16(21, 1500, P(s), P(ys))
    out.update(lsm_y=ys.copy())
    # activations (positive-domain kinds get |x| + 0.1)
    a, ap = gi["act_x"], gi["act_xp"]
    for k in oracle.ACT_KINDS:
        src = ap if k in oracle.POSITIVE_KINDS else a
        ya = np.empty_like(src)
        L.rocket_activation_ref_fp16(k, P(src), P(ya), src.size)
        out[f"act_y{k}"] = ya.copy()
    # mha (T=40, d=128, 2 heads of 64)
    p = gi["mha"]
    ym = np.empty((40, 128), np.float16)
    L.rocket_mha_self_ref_fp16(40, 128, 2, P(p["x"]), P(p["Wq"]), P(p["bq"]), P(p["Wk"]), P(p["bk"]),
                               P(p["Wv"]), P(p["bv"]), P(p["Wo"]), P(p["bo"]), P(ym))
    out.update(mha_y=ym)
    # ffn (M=16, H=128, I=256), GELU and SiLU
    fx, Wg, Wu, Wd = gi["ffn_x"], gi["ffn_Wg"], gi["ffn_Wu"], gi["ffn_Wd"]
    for kind in (3, 5):
        yf = np.empty((16, 128), np.float16)
        L.rocket_ffn_ref_fp16(16, 128, 256, P(fx), P(Wg), P(Wu), P(Wd), kind, P(yf))
        out[f"ffn_y{kind}"] = yf
    # encoder block at the reference gate's first shape (64, 256, 4, 1024)
    p = gi["enc"]
    ye = np.empty((64, 256), np.float16)
    keys = ["ln1_g", "ln1_b", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo", "ln2_g", "ln2_b",
            "W1", "b1", "W2", "b2"]
    L.rocket_encoder_block_ref_fp16(64, 256, 4, 1024, P(p["x"]), *[P(p[k]) for k in keys], F(1e-5), P(ye))
    out.update(enc_y=ye)
    np.savez_compressed(os.path.join(HERE, "encoder_golden.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
