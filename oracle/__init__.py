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
def rel_frobenius(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-300))


def max_abs_rel(got, ref):
    """max |got - ref| / max |ref| (the north-star's max-abs relative error)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-300))
