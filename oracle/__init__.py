"""TEST INFRASTRUCTURE ONLY: ctypes front-end of liboracle.so.

The oracle is a CPU restatement of the reference's host computations
(oracle.c, each function citing the reference test it follows), pinned by
running the reference's own gates against it (oracle/Makefile `pin`).  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


def _load():
    if not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True, capture_output=True)
    lib = ctypes.CDLL(LIB_PATH)
    P, I, U64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_float
    sigs = {
        "orc_glibc_i8": (None, [ctypes.c_uint, I, I, ctypes.c_size_t, P]),
        "orc_uniform_i8": (None, [U64, I, I, ctypes.c_size_t, P]),
        "orc_uniform_f32": (None, [U64, F, F, ctypes.c_size_t, P]),
        "orc_normal_f16": (None, [U64, F, ctypes.c_size_t, P]),
        "orc_normal_f32": (None, [U64, F, F, ctypes.c_size_t, P]),
        "orc_matmul_int8": (None, [I, I, I, P, P, P, I, I, I]),
        "orc_matmul_fp16": (None, [I, I, I, P, P, P, P, I, I, I]),
        "orc_gw_ref": (None, [I, I, I, I, P, P, P, P, P, I, I, I]),
        "orc_gw_f32": (None, [I, I, I, I, P, P, P, P, P]),
    }
    for n, (r, a) in sigs.items():
        fn = getattr(lib, n)
        fn.restype = r
        fn.argtypes = a
    return lib


lib = _load()


def _p(a):
    return None if a is None else a.ctypes.data


# ---- generators (seeded, deterministic) ----
def uniform_i8(seed, lo, hi, shape):
    out = np.empty(shape, np.int8)
    lib.orc_uniform_i8(seed, lo, hi, out.size, _p(out))
    return out


def uniform_f32(seed, lo, hi, shape):
    out = np.empty(shape, np.float32)
    lib.orc_uniform_f32(seed, lo, hi, out.size, _p(out))
    return out


def normal_f16(seed, scale, shape):
    out = np.empty(shape, np.float16)
    lib.orc_normal_f16(seed, scale, out.size, _p(out))
    return out


def normal_f32(seed, mean, std, shape):
    out = np.empty(shape, np.float32)
    lib.orc_normal_f32(seed, mean, std, out.size, _p(out))
    return out


def glibc_i8(seed, lo, span, shape):
    out = np.empty(shape, np.int8)
    lib.orc_glibc_i8(seed, lo, span, out.size, _p(out))
    return out


# ---- restatements ----
def matmul_int8(A, B, rows=None, nthreads=1):
    M, K = A.shape
    N = B.shape[0]
    r0, r1 = (0, M) if rows is None else rows
    C = np.zeros((M, N), np.int32)
    lib.orc_matmul_int8(M, K, N, _p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(B)), _p(C), r0, r1, nthreads)
    return C


def matmul_fp16(A, B, rows=None, nthreads=1):
    """Returns (fp32 sum, fp16-narrowed result)."""
    M, K = A.shape
    N = B.shape[0]
    r0, r1 = (0, M) if rows is None else rows
    R = np.zeros((M, N), np.float32)
    C = np.zeros((M, N), np.float16)
    lib.orc_matmul_fp16(M, K, N, _p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(B)), _p(R), _p(C),
                        r0, r1, nthreads)
    return R, C


def gw_ref(A, B, a_scale, b_scale, group, rows=None, nthreads=1):
    M, K = A.shape
    N = B.shape[0]
    r0, r1 = (0, M) if rows is None else rows
    ref = np.zeros((M, N), np.float64)
    lib.orc_gw_ref(M, K, N, group, _p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(B)),
                   _p(np.ascontiguousarray(a_scale, np.float32)), _p(np.ascontiguousarray(b_scale, np.float32)),
                   _p(ref), r0, r1, nthreads)
    return ref


def gw_f32(A, B, a_scale, b_scale, group):
    M, K = A.shape
    N = B.shape[0]
    C = np.zeros((M, N), np.float32)
    lib.orc_gw_f32(M, K, N, group, _p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(B)),
                   _p(np.ascontiguousarray(a_scale, np.float32)), _p(np.ascontiguousarray(b_scale, np.float32)),
                   _p(C))
    return C


# ---- tolerance metrics used by the parity tests ----
def rms_normalised_err(got, ref):
    """max |got - ref| / rms(ref): the reference's group-wise gates bound this
    by 1e-5 (tests/matmul_int8_groupwise_rocket.c:59-82)."""
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref)))
    d = np.abs(np.asarray(got, np.float64) - ref)
    return float(d.max()) / rms if rms > 0 else float(d.max())


def rel_frobenius(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-300))


def max_abs_rel(got, ref):
    """max |got - ref| / max |ref| (the north-star's max-abs relative error)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-300))


# ---- encoder ops ----
def _sig_enc():
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    sigs = {
        "orc_layernorm_f16": [I, I, P, P, P, F, P],
        "orc_rmsnorm_f16": [I, I, P, P, F, P],
        "orc_softmax_f16": [I, I, P, I, P],
        "orc_activation_f16": [I, P, P, ctypes.c_size_t],
        "orc_mha_self_f16": [I, I, I] + [P] * 10,
        "orc_ffn_f16": [I, I, I, P, P, P, P, I, P],
        "orc_encoder_block_f16": [I, I, I, I] + [P] * 17 + [F, P],
    }
    for n, a in sigs.items():
        getattr(lib, n).restype = None
        getattr(lib, n).argtypes = a


_sig_enc()


def _h(a):
    return None if a is None else np.ascontiguousarray(a, np.float16).ctypes.data


def layernorm(x, g, b, eps):
    M, H = x.shape
    y = np.empty_like(x, dtype=np.float16)
    lib.orc_layernorm_f16(M, H, _h(x), _h(g), _h(b), eps, y.ctypes.data)
    return y


def rmsnorm(x, w, eps):
    M, H = x.shape
    y = np.empty_like(x, dtype=np.float16)
    lib.orc_rmsnorm_f16(M, H, _h(x), _h(w), eps, y.ctypes.data)
    return y


def softmax(x, log_mode=False):
    M, N = x.shape
    y = np.empty_like(x, dtype=np.float16)
    lib.orc_softmax_f16(M, N, _h(x), int(log_mode), y.ctypes.data)
    return y


def activation(kind, x):
    y = np.empty_like(x, dtype=np.float16)
    lib.orc_activation_f16(kind, _h(x), y.ctypes.data, x.size)
    return y


def mha_self(x, Wq, bq, Wk, bk, Wv, bv, Wo, bo, n_head):
    T, d = x.shape
    y = np.empty((T, d), np.float16)
    lib.orc_mha_self_f16(T, d, n_head, _h(x), _h(Wq), _h(bq), _h(Wk), _h(bk), _h(Wv), _h(bv),
                         _h(Wo), _h(bo), y.ctypes.data)
    return y


def ffn(x, Wg, Wu, Wd, kind):
    M, H = x.shape
    I = Wg.shape[0]
    y = np.empty((M, H), np.float16)
    lib.orc_ffn_f16(M, H, I, _h(x), _h(Wg), _h(Wu), _h(Wd), kind, y.ctypes.data)
    return y


def encoder_block(x, p, n_head, eps=1e-5):
    """p: dict of ln1_g ln1_b Wq bq Wk bk Wv bv Wo bo ln2_g ln2_b W1 b1 W2 b2 (fp16 arrays)."""
    T, d = x.shape
    dff = p["W1"].shape[0]
    y = np.empty((T, d), np.float16)
    keys = ["ln1_g", "ln1_b", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo", "ln2_g", "ln2_b",
            "W1", "b1", "W2", "b2"]
    lib.orc_encoder_block_f16(T, d, n_head, dff, _h(x), *[_h(p.get(k)) for k in keys], eps, y.ctypes.data)
    return y


def encoder_params(T, d, nh, dff, seed):
    """Seeded encoder-block inputs: x ~ N(0,1), weights and biases ~ N(0, 0.02),
    LN gamma = 1, beta = 0 (the BASELINE config-4 distributions)."""
    p = {"x": normal_f16(seed, 1.0, (T, d)),
         "ln1_g": np.ones(d, np.float16), "ln1_b": np.zeros(d, np.float16),
         "ln2_g": np.ones(d, np.float16), "ln2_b": np.zeros(d, np.float16)}
    for i, (k, shp) in enumerate([("Wq", (d, d)), ("Wk", (d, d)), ("Wv", (d, d)), ("Wo", (d, d)),
                                  ("W1", (dff, d)), ("W2", (d, dff))]):
        p[k] = normal_f16(seed + 10 + i, 0.02, shp)
    for i, (k, n) in enumerate([("bq", d), ("bk", d), ("bv", d), ("bo", d), ("b1", dff), ("b2", d)]):
        p[k] = normal_f16(seed + 30 + i, 0.02, (n,))
    return p


def encoder_golden_inputs():
    """The seeded inputs of tests/golden/encoder_golden.npz (outputs only are stored)."""
    d = {}
    d["ln_x"] = normal_f16(101, 2.0, (37, 512))
    d["ln_g"] = normal_f16(102, 1.0, (512,))
    d["ln_b"] = normal_f16(103, 0.5, (512,))
    d["sm_x"] = normal_f16(104, 3.0, (21, 1500))
    a = normal_f16(105, 3.0, (4096,))
    d["act_x"] = a
    d["act_xp"] = (np.abs(a.astype(np.float32)) + 0.1).astype(np.float16)
    d["mha"] = encoder_params(40, 128, 2, 256, 200)
    d["ffn_x"] = normal_f16(300, 1.0, (16, 128))
    d["ffn_Wg"] = normal_f16(301, 0.05, (256, 128))
    d["ffn_Wu"] = normal_f16(302, 0.05, (256, 128))
    d["ffn_Wd"] = normal_f16(303, 0.05, (128, 256))
    d["enc"] = encoder_params(64, 256, 4, 1024, 400)
    return d


ACT_KINDS = [0, 1, 2, 3, 4, 5, 7, 8, 9, 10, 11, 12, 13, 14, 15, 18]
POSITIVE_KINDS = (7, 8, 9, 18)


# ---- reductions (oracle.c, bit-exact restatements of the reference's host refs) ----
def _sig_red():
    P, I = ctypes.c_void_p, ctypes.c_int
    for n, a in {"orc_reduce_feature_f16": [I, I, P, I, P], "orc_cumsum_f16": [I, I, P, I, I, P],
                 "orc_scale_rows_f16": [I, I, P, P, P], "orc_cross_entropy_f16": [I, I, P, P, P]}.items():
        getattr(lib, n).restype = None
        getattr(lib, n).argtypes = a


_sig_red()


def reduce_feature(x, mean=False):
    M, H = x.shape
    out = np.empty(M, np.float32)
    lib.orc_reduce_feature_f16(M, H, _h(x), int(mean), out.ctypes.data)
    return out


def cumsum(x, exclusive=False, reverse=False):
    M, N = x.shape
    y = np.empty((M, N), np.float16)
    lib.orc_cumsum_f16(M, N, _h(x), int(exclusive), int(reverse), y.ctypes.data)
    return y


def scale_rows(x, r):
    M, N = x.shape
    y = np.empty((M, N), np.float16)
    lib.orc_scale_rows_f16(M, N, _h(x), np.ascontiguousarray(r, np.float32).ctypes.data, y.ctypes.data)
    return y


def cross_entropy(x, target):
    M, N = x.shape
    loss = np.empty(M, np.float32)
    lib.orc_cross_entropy_f16(M, N, _h(x), np.ascontiguousarray(target, np.int32).ctypes.data,
                              loss.ctypes.data)
    return loss


# ---- dtype matmuls (C = A . B^T, fp64 references) ----
def bf16_trunc(a):
    """fp32 -> bf16 -> fp32 by dropping the low 16 bits (src/rocket_matmul.c:3456-3458)."""
    return (np.ascontiguousarray(a, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


def matmul_bf16(A, B):
    """Truncated-bf16 products accumulated in fp64 (tests/matmul_bf16_tiled_rocket.c ref)."""
    return bf16_trunc(A).astype(np.float64) @ bf16_trunc(B).astype(np.float64).T


def matmul_f64(A, B):
    """fp64 product of the raw inputs (the tf32 and fp16->fp32 gates' reference)."""
    return np.asarray(A, np.float64) @ np.asarray(B, np.float64).T


def int16_clamp(a):
    """The exact int16 route's input domain [-32768, 32639] (src/rocket_matmul.c:3397-3403)."""
    return np.clip(np.asarray(a, np.int64), -32768, 32639)


def matmul_int16_exact(A, B):
    """int64 A . B^T over the clamped inputs (bit-exact target)."""
    return int16_clamp(A) @ int16_clamp(B).T


def reduce_golden_inputs():
    """Seeded inputs of tests/golden/reduce_golden.npz: x [37, 300] fp16 ~ N(0, 1)
    (ragged: neither dimension a multiple of 32), per-row scales r [37], logits
    [33, 1000] ~ N(0, 3) with targets that include -1 and N (out of range)."""
    x = normal_f16(71, 1.0, (37, 300))
    r = uniform_f32(72, -2.0, 2.0, (37,))
    logits = normal_f16(73, 3.0, (33, 1000))
    t = (np.arange(33, dtype=np.int64) * 397 % 1000).astype(np.int32)
    t[5], t[11] = -1, 1000
    return {"x": x, "r": r, "logits": logits, "target": t}


# ---- masked grouped-query attention ----
lib.orc_flash_attn_f16.restype = None
lib.orc_flash_attn_f16.argtypes = [ctypes.c_int] * 6 + [ctypes.c_float] * 2 + [ctypes.c_void_p] * 5


def flash_attn(Q, K, V, mask, scale, softcap=0.0):
    """Q [nh, T, dh], K [nkvh, n_kv, dh], V [nkvh, dv, n_kv], mask [T, n_kv] or None."""
    nh, T, dh = Q.shape
    nkvh, n_kv, _ = K.shape
    dv = V.shape[1]
    out = np.empty((nh, T, dv), np.float16)
    lib.orc_flash_attn_f16(T, n_kv, dh, dv, nh, nkvh, scale, softcap, _h(Q), _h(K), _h(V), _h(mask),
                           out.ctypes.data)
    return out


def causal_mask(T, n_kv, window=0):
    """Additive causal (+ sliding window) mask [T, n_kv] with keys aligned to the
    tail of the cache (tests/flash_attn_rocket.c:44-52 convention): 0 kept, -inf masked."""
    pos = n_kv - T + np.arange(T)[:, None]
    j = np.arange(n_kv)[None, :]
    keep = (j <= pos) & ((window <= 0) | (j > pos - window))
    return np.where(keep, 0.0, -np.inf).astype(np.float16)


# (T, n_kv, dh, dv, nh, nkvh, window, softcap): the reference gate's cases, scaled down
FA_GOLDEN_CASES = [
    (32, 32, 64, 64, 4, 2, 0, 0.0),
    (20, 45, 96, 96, 4, 1, 8, 0.0),
    (16, 64, 192, 128, 2, 1, 0, 0.0),
    (24, 24, 128, 128, 2, 2, 0, 50.0),
    (8, 40, 256, 256, 2, 1, 0, 0.0),
]


def fa_golden_inputs(case):
    T, n_kv, dh, dv, nh, nkvh, window, _ = case
    seed = T * 1000 + n_kv * 10 + dh
    Q = normal_f16(seed + 1, 1.0, (nh, T, dh))
    K = normal_f16(seed + 2, 1.0, (nkvh, n_kv, dh))
    V = normal_f16(seed + 3, 1.0, (nkvh, dv, n_kv))
    return Q, K, V, causal_mask(T, n_kv, window)
