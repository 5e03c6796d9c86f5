"""Python host mirror of librocketnpu (B200 build).

ctypes bindings over ``librocketnpu.so`` -- the C-ABI library whose headers
are ``include/rocket_npu.h`` and ``include/rocket_matmul.h``.  Function names,
argument meaning and return codes are the reference's (gregordinary/
rocket-userspace ``include/rocket_matmul.h``); the thin wrappers below only
convert numpy arrays / torch tensors to pointers.  There is no fallback: if
the shared library is missing, importing this module raises.

Pointers may be host memory (numpy arrays, CPU tensors) or device memory
(CUDA tensors on the handle's GPU), exactly as the C entry points accept.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int8, c_int32, c_long, c_size_t, c_uint64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ROCKET_LIB_PATH") or os.path.join(_HERE, "librocketnpu.so")

ROCKET_OK = 0
ROCKET_E_SHAPE = -1
ROCKET_E_TILING = -2
ROCKET_E_NOMEM = -3
ROCKET_E_DEVICE = -4
ROCKET_E_UNSUPPORTED = -5

# (name, restype, argtypes) for every symbol the public headers declare.
_P = c_void_p
_SIGS = [
    # rocket_npu.h
    ("rocket_open", c_int, []),
    ("rocket_close", None, [c_int]),
    ("rocket_affinity_set_base", None, [c_int]),
    ("rocket_affinity_get_base", c_int, []),
    ("rocket_pin_worker", None, [c_int]),
    ("rocket_num_big_cores", c_int, []),
    ("rocket_bo_alloc", c_int, [c_int, c_size_t, _P]),
    ("rocket_bo_free", None, [c_int, _P]),
    ("rocket_bo_prep", c_int, [c_int, _P, c_int, c_uint64]),
    ("rocket_bo_fini", c_int, [c_int, _P]),
    ("rocket_bo_prep_ranges", c_int, [c_int, _P, _P, ctypes.c_uint, c_uint64]),
    ("rocket_bo_fini_ranges", c_int, [c_int, _P, _P, ctypes.c_uint]),
    ("rocket_bo_ranges_supported", c_int, []),
    ("rocket_batched_submit_supported", c_int, []),
    ("rocket_ppu_done_supported", c_int, []),
    ("rocket_batch_completion_tracked", c_int, []),
    ("rocket_busy_poll_set_us", None, [c_long]),
    ("rocket_submit_matmul", c_int, [c_int, _P, ctypes.c_uint32, _P, ctypes.c_uint32, _P, ctypes.c_uint32, ctypes.c_uint32]),
    ("rocket_submit_matmul_flags", c_int, [c_int, _P, ctypes.c_uint32, _P, ctypes.c_uint32, _P, ctypes.c_uint32, ctypes.c_uint32]),
    ("rocket_submit_tasks", c_int, [c_int, _P, ctypes.c_uint32, _P, ctypes.c_uint32, _P, ctypes.c_uint32]),
    ("rocket_submit_tasks_flags", c_int, [c_int, _P, ctypes.c_uint32, _P, ctypes.c_uint32, _P, ctypes.c_uint32, ctypes.c_uint32]),
    ("rocket_submit_scratch_size", c_size_t, [ctypes.c_uint32]),
    ("rocket_submit_tasks_pre", c_int, [c_int, _P, _P, ctypes.c_uint32, _P, ctypes.c_uint32, _P, ctypes.c_uint32, ctypes.c_uint32]),
    ("rocket_submit_jobs", c_int, [c_int, _P, ctypes.c_uint32]),
    ("rocket_submit_ioctl_count", c_uint64, []),
    ("rocket_submit_task_count", c_uint64, []),
    ("rocket_submit_counters_reset", None, []),
    # rocket_log.h
    ("rocket_log_set_callback", None, [_P, _P]),
    ("rocket_log_set_level", None, [c_int]),
    ("rocket_log_get_level", c_int, []),
    # rocket_matmul.h
    ("rocket_matmul_plan", c_int, [c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_plan_int8", c_int, [c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_plan_int8_gw", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_plan_int4", c_int, [c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_fp16", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_int8", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_int8_groupwise", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, c_int]),
    ("rocket_matmul_int4", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_int4_ex", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P, c_int]),
    ("rocket_matmul_int4_groupwise", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, c_int]),
    ("rocket_matmul_fp16_mt", c_int, [c_int, c_int, c_int, _P, _P, _P, c_int]),
    ("rocket_ctx_create", _P, [c_int]),
    ("rocket_ctx_free", None, [_P]),
    ("rocket_weights_pack", _P, [_P, c_int, c_int, c_int, _P]),
    ("rocket_weights_free", None, [_P, _P]),
    ("rocket_matmul_fp16_prepacked", c_int, [_P, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_i8_ctx_create", _P, [c_int]),
    ("rocket_i8_ctx_free", None, [_P]),
    ("rocket_i8_weights_pack", _P, [_P, c_int, c_int, c_int, _P]),
    ("rocket_i8_weights_pack_gw", _P, [_P, c_int, c_int, c_int, _P, c_int]),
    ("rocket_i8_weights_free", None, [_P, _P]),
    ("rocket_i8_weights_bytes", c_size_t, [_P]),
    ("rocket_matmul_int8_prepacked", c_int, [_P, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_int8_prepacked_gw", c_int, [_P, c_int, c_int, c_int, _P, _P, _P, _P, _P]),
    ("rocket_i4_ctx_create", _P, [c_int]),
    ("rocket_i4_ctx_free", None, [_P]),
    ("rocket_i4_weights_pack", _P, [_P, c_int, c_int, c_int, _P]),
    ("rocket_i4_weights_pack_gw", _P, [_P, c_int, c_int, c_int, _P, c_int]),
    ("rocket_i4_weights_free", None, [_P, _P]),
    ("rocket_i4_weights_bytes", c_size_t, [_P]),
    ("rocket_matmul_int4_prepacked", c_int, [_P, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_int4_prepacked_gw", c_int, [_P, c_int, c_int, c_int, _P, _P, _P, _P, _P]),
]

# rocket_b200.h extensions (no reference counterpart)
_SIGS += [
    ("rocket_b200_stream", c_void_p, [c_int]),
    ("rocket_b200_device", c_int, [c_int]),
    ("rocket_b200_ctx_fd", c_int, [c_void_p, c_int]),
    ("rocket_b200_profile_enable", None, [c_int]),
    ("rocket_b200_profile_reset", None, []),
    ("rocket_b200_profile_get", c_int, [c_int, POINTER(c_char_p), POINTER(c_uint64), POINTER(ctypes.c_double)]),
    ("rocket_b200_set_async", None, [c_int]),
    ("rocket_b200_sync", c_int, [c_int]),
    ("rocket_b200_ctx_sync", c_int, [c_void_p]),
    ("rocket_b200_matmul_int4_groupwise_noalloc", c_int,
     [c_int, c_int, c_int, _P, _P, _P, _P, _P, c_int, _P]),
]

# encoder ops: rocket_norm.h, rocket_softmax.h, rocket_activation.h, rocket_ffn.h,
# rocket_attn.h, rocket_encoder.h (+ the batched rocket_b200.h form)
_F = ctypes.c_float
_SIGS += [
    ("rocket_layernorm_fp16", c_int, [c_int, c_int, c_int, _P, _P, _P, _F, _P]),
    ("rocket_rmsnorm_fp16", c_int, [c_int, c_int, c_int, _P, _P, _F, _P]),
    ("rocket_softmax_fp16", c_int, [c_int, c_int, c_int, _P, _P]),
    ("rocket_logsoftmax_fp16", c_int, [c_int, c_int, c_int, _P, _P]),
    ("rocket_activation_fp16", c_int, [c_int, c_int, _P, _P, c_int]),
    ("rocket_ew_mul_fp16", c_int, [c_int, _P, _P, _P, c_int]),
    ("rocket_ew_add_fp16", c_int, [c_int, _P, _P, _P, c_int]),
    ("rocket_ew_sub_fp16", c_int, [c_int, _P, _P, _P, c_int]),
    ("rocket_ew_max_fp16", c_int, [c_int, _P, _P, _P, c_int]),
    ("rocket_ew_min_fp16", c_int, [c_int, _P, _P, _P, c_int]),
    ("rocket_clip_fp16", c_int, [c_int, c_float, c_float, _P, _P, c_int]),
    ("rocket_activation_name", c_char_p, [c_int]),
    # rocket_hw_profile.h
    ("rocket_hw_current", c_void_p, []),
    ("rocket_hw_by_name", c_void_p, [c_char_p]),
    ("rocket_geglu_fp16", c_int, [c_int, _P, _P, c_int, _P, c_int]),
    ("rocket_ffn_fp16", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, _P]),
    ("rocket_ffn_fp16_fused", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, _P]),
    ("rocket_mlp_fp16_fused", c_int, [c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, _P]),
    ("rocket_mha_self_fp16", c_int, [c_int, c_int, c_int, c_int] + [_P] * 10),
    ("rocket_encoder_block_fp16", c_int, [c_int, c_int, c_int, c_int, c_int] + [_P] * 17 + [_F, _P]),
    ("rocket_b200_encoder_block_batched_fp16", c_int,
     [c_int, c_int, c_int, c_int, c_int, c_int] + [_P] * 17 + [_F, _P]),
]

_SIGS += [
    ("rocket_reduce_feature_fp16", c_int, [c_int, c_int, c_int, _P, _P, c_int]),
    ("rocket_cumsum_fp16", c_int, [c_int, c_int, c_int, _P, _P, c_int, c_int]),
    ("rocket_scale_rows_fp16", c_int, [c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_cross_entropy_fp16", c_int, [c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_fp16_f32out", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_fp16_batch", c_int, [c_int, c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_mm_batch_create", _P, [c_int]),
    ("rocket_mm_batch_free", None, [_P]),
    ("rocket_mm_batch_run", c_int, [_P, c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_plan_int16", c_int, [c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_int16_exact", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_plan_bf16", c_int, [c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_bf16", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_bf16_mt", c_int, [c_int, c_int, c_int, _P, _P, _P, c_int]),
    ("rocket_bf16_stream_create", _P, [c_int]),
    ("rocket_bf16_stream_free", None, [_P]),
    ("rocket_matmul_bf16_stream", c_int, [_P, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_plan_tf32", c_int, [c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_tf32", c_int, [c_int, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_stream_create", _P, [c_int]),
    ("rocket_stream_free", None, [_P]),
    ("rocket_matmul_fp16_stream", c_int, [_P, c_int, c_int, c_int, _P, _P, _P]),
    ("rocket_matmul_fp16_stream_fused", c_int, [_P, c_int, c_int, _P, _P, c_int, _P, _P]),
    ("rocket_b200_gemm_policy", c_int, [c_int, c_int]),
    ("rocket_b200_gw_mode", c_int, [c_int]),
    ("rocket_fa_ctx_create", _P, [c_int]),
    ("rocket_fa_ctx_free", None, [_P]),
    ("rocket_flash_attn_fp16", c_int, [c_int] * 7 + [c_float, c_float] + [_P] * 5),
    ("rocket_flash_attn_fp16_mt", c_int, [c_int] * 7 + [c_float, c_float] + [_P] * 5 + [c_int]),
    ("rocket_flash_attn_fp16_ctx", c_int, [_P] + [c_int] * 6 + [c_float, c_float] + [_P] * 5),
]

ENCODER_KEYS = ["ln1_g", "ln1_b", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo", "ln2_g", "ln2_b",
                "W1", "b1", "W2", "b2"]

EXTRA_SIGS: list = []


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"librocketnpu.so not built at {LIB_PATH}: run `make -C rocket-userspace_b200` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, res, args in _SIGS:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

def _load_shard():
    import importlib.util
    spec = importlib.util.spec_from_file_location(__name__ + ".shard", os.path.join(_HERE, "shard.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


shard = _load_shard()   # N-column sharding across ranks


def declared_symbols() -> list[str]:
    return [n for n, _, _ in _SIGS]


# ---------------------------------------------------------------- pointer glue
def ptr(x) -> int:
    """Address of a numpy array or torch tensor (contiguous), or 0 for None."""
    if x is None:
        return 0
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("array must be C-contiguous")
        return x.ctypes.data
    raise TypeError(type(x))


class Device:
    """An open device handle (rocket_open / rocket_close)."""

    def __init__(self):
        self.fd = lib.rocket_open()
        if self.fd < 0:
            raise RuntimeError(f"rocket_open failed ({self.fd})")

    def close(self):
        if self.fd >= 0:
            lib.rocket_close(self.fd)
            self.fd = -1

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # one-shot entries; return the rocket_status
    def matmul_fp16(self, M, K, N, A, B, C):
        return lib.rocket_matmul_fp16(self.fd, M, K, N, ptr(A), ptr(B), ptr(C))

    def matmul_int8(self, M, K, N, A, B, C):
        return lib.rocket_matmul_int8(self.fd, M, K, N, ptr(A), ptr(B), ptr(C))

    def matmul_int4(self, M, K, N, A, B, C, kt_cap=0):
        return lib.rocket_matmul_int4_ex(self.fd, M, K, N, ptr(A), ptr(B), ptr(C), kt_cap)

    def matmul_int8_groupwise(self, M, K, N, A, B, a_scale, b_scale, Cf, group):
        return lib.rocket_matmul_int8_groupwise(self.fd, M, K, N, ptr(A), ptr(B), ptr(a_scale),
                                                ptr(b_scale), ptr(Cf), group)

    def matmul_int4_groupwise(self, M, K, N, A, B, a_scale, b_scale, Cf, group):
        return lib.rocket_matmul_int4_groupwise(self.fd, M, K, N, ptr(A), ptr(B), ptr(a_scale),
                                                ptr(b_scale), ptr(Cf), group)


def profile_snapshot() -> dict:
    """{family: (launches, total_ms)} from the library's kernel profiler."""
    out = {}
    i = 0
    name, n, ms = c_char_p(), c_uint64(), ctypes.c_double()
    while lib.rocket_b200_profile_get(i, ctypes.byref(name), ctypes.byref(n), ctypes.byref(ms)) == 0:
        out[name.value.decode()] = (n.value, ms.value)
        i += 1
    return out


def plan(kind: str, M, K, N, group=None):
    mt, kt, nt = c_int(), c_int(), c_int()
    r = ctypes.byref
    if kind == "fp16":
        rc = lib.rocket_matmul_plan(M, K, N, r(mt), r(kt), r(nt))
    elif kind == "int8":
        rc = lib.rocket_matmul_plan_int8(M, K, N, r(mt), r(kt), r(nt))
    elif kind == "int8_gw":
        rc = lib.rocket_matmul_plan_int8_gw(M, K, N, group, r(mt), r(kt), r(nt))
    elif kind == "int4":
        rc = lib.rocket_matmul_plan_int4(M, K, N, r(mt), r(kt), r(nt))
    else:
        raise ValueError(kind)
    return rc, (mt.value, kt.value, nt.value)
