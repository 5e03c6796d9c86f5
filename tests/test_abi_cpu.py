"""CPU: the C-ABI library loads, exports every function include/*.h declares,
and its host-side logic (tiling previews, shape rules, no-device behaviour)
follows the reference's contract without touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(REPO, "include")


def declared_functions():
    names = set()
    for h in sorted(os.listdir(INCLUDE)):
        if not h.endswith(".h"):
            continue
        src = open(os.path.join(INCLUDE, h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"#define[^\n]*", "", src)
        for m in re.finditer(r"\b(rocket_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_hot_path():
    names = declared_functions()
    for must in ["rocket_open", "rocket_close", "rocket_matmul_fp16", "rocket_matmul_int8",
                 "rocket_matmul_int8_groupwise", "rocket_matmul_int4", "rocket_matmul_int4_ex",
                 "rocket_matmul_int4_groupwise", "rocket_matmul_fp16_mt", "rocket_ctx_create",
                 "rocket_weights_pack", "rocket_matmul_fp16_prepacked", "rocket_i8_ctx_create",
                 "rocket_i8_weights_pack_gw", "rocket_matmul_int8_prepacked_gw",
                 "rocket_i4_weights_pack_gw", "rocket_matmul_int4_prepacked_gw", "rocket_log"]:
        assert must in names


def test_library_exports_every_declared_symbol(rkb):
    lib = ctypes.CDLL(rkb.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python mirror binds every one of them
    bound = set(rkb.declared_symbols()) | {n for n, _, _ in rkb.EXTRA_SIGS} | {"rocket_log"}
    assert not [n for n in declared_functions() if n not in bound]


def test_library_links_no_torch_and_no_oracle(rkb):
    out = subprocess.run(["ldd", rkb.LIB_PATH], capture_output=True, text=True).stdout
    assert "torch" not in out and "oracle" not in out
    syms = subprocess.run(["nm", "-D", rkb.LIB_PATH], capture_output=True, text=True).stdout
    assert "orc_" not in syms


@pytest.mark.parametrize("kind,M,K,N,ok", [
    ("fp16", 512, 4096, 4096, True), ("fp16", 1, 64, 48, True), ("fp16", 6, 64, 48, False),
    ("fp16", 8, 48, 48, False), ("fp16", 8, 64, 40, False),
    ("int8", 64, 512, 256, True), ("int8", 64, 512, 48, False), ("int8", 4096, 3840, 5888, True),
    ("int4", 64, 512, 256, True), ("int4", 64, 512, 96, False),
])
def test_plan_shape_rules(rkb, kind, M, K, N, ok):
    rc, (mt, kt, nt) = rkb.plan(kind, M, K, N)
    if ok:
        assert rc > 0
        assert rc == ((M + 127) // 128) * ((N + 255) // 256)
        assert 0 < mt <= 128 and 0 < nt <= 256 and 0 < kt <= K
    else:
        assert rc == rkb.ROCKET_E_SHAPE


def test_plan_groupwise_rules(rkb):
    assert rkb.plan("int8_gw", 64, 3840, 256, group=32)[0] > 0
    assert rkb.plan("int8_gw", 64, 3840, 256, group=48)[0] == rkb.ROCKET_E_SHAPE   # not %32
    assert rkb.plan("int8_gw", 64, 3840, 256, group=512)[0] == rkb.ROCKET_E_SHAPE  # does not divide K
    assert rkb.plan("int8_gw", 1, 3840, 256, group=32)[0] == rkb.ROCKET_E_SHAPE    # gw: M%4 only


def test_bad_shapes_rejected_before_device(rkb):
    import numpy as np
    A = np.zeros((6, 64), np.int8)
    B = np.zeros((32, 64), np.int8)
    C = np.zeros((6, 32), np.int32)
    # shape check happens before the handle is looked up
    assert rkb.lib.rocket_matmul_int8(0, 6, 64, 32, rkb.ptr(A), rkb.ptr(B), rkb.ptr(C)) == rkb.ROCKET_E_SHAPE


def test_no_device_behaviour(rkb):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    assert rkb.lib.rocket_open() == rkb.ROCKET_E_DEVICE
    assert rkb.lib.rocket_i8_ctx_create(2) is None
    assert rkb.lib.rocket_ctx_create(1) is None
    assert rkb.lib.rocket_i4_ctx_create(1) is None


def test_submit_family_unsupported(rkb):
    assert rkb.lib.rocket_submit_tasks(0, None, 0, None, 0, None, 0) == rkb.ROCKET_E_UNSUPPORTED
    assert rkb.lib.rocket_submit_jobs(0, None, 0) == rkb.ROCKET_E_UNSUPPORTED
    assert rkb.lib.rocket_batched_submit_supported() == 0
    assert rkb.lib.rocket_bo_ranges_supported() == 1


def test_affinity_and_counters(rkb):
    rkb.lib.rocket_affinity_set_base(6)
    assert rkb.lib.rocket_affinity_get_base() == 6
    rkb.lib.rocket_affinity_set_base(0)
    assert rkb.lib.rocket_num_big_cores() == 0
    rkb.lib.rocket_submit_counters_reset()
    assert rkb.lib.rocket_submit_ioctl_count() == 0


def test_log_callback_and_level(rkb):
    seen = []
    CB = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p)
    cb = CB(lambda lvl, txt, ud: seen.append((lvl, txt.decode())))
    rkb.lib.rocket_log_set_callback(ctypes.cast(cb, ctypes.c_void_p), None)
    try:
        rkb.lib.rocket_log_set_level(3)
        assert rkb.lib.rocket_log_get_level() == 3
        import numpy as np
        A = np.zeros((6, 64), np.int8)
        rkb.lib.rocket_matmul_int8(0, 6, 64, 32, rkb.ptr(A), rkb.ptr(A), rkb.ptr(A))
        assert any("bad shape" in t for _, t in seen)
    finally:
        rkb.lib.rocket_log_set_callback(None, None)
        rkb.lib.rocket_log_set_level(2)


@pytest.mark.parametrize("group,kt", [(32, 32), (96, 96), (576, 576), (1024, 1024), (1440, 1440),
                                      (2880, 2880), (2048, 2048)])
def test_plan_int8_gw_kt_is_exact_partial_length(rkb, group, kt):
    """Kt of the group-wise plan is the K per exact integer partial of the
    precise kernel: the whole group, since int32 partials are exact for any
    group (|a w| <= 2^14)."""
    Mt, Kt, Nt = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    K = group * 2 if group < 2880 else 2880
    rc = rkb.lib.rocket_matmul_plan_int8_gw(128, K, 256, group, ctypes.byref(Mt), ctypes.byref(Kt),
                                            ctypes.byref(Nt))
    assert rc > 0
    assert Kt.value == kt


def test_hw_profile_layout(rkb):
    """rocket_hw_current() follows the reference's struct layout
    (include/rocket_hw_profile.h): the gates read max_tile from it."""
    class Prof(ctypes.Structure):
        _fields_ = [("name", ctypes.c_char_p), ("cbuf_banks", ctypes.c_int), ("cbuf_bank_size", ctypes.c_int),
                    ("max_tile", ctypes.c_int), ("kgroup_2b", ctypes.c_int), ("kgroup_4b", ctypes.c_int),
                    ("ngroup", ctypes.c_int), ("dtype_supported", ctypes.c_uint32),
                    ("select_warning", ctypes.c_char_p), ("default_workers", ctypes.c_int)]
    p = ctypes.cast(rkb.lib.rocket_hw_current(), ctypes.POINTER(Prof)).contents
    assert p.name == b"b200" and p.max_tile == 256 and p.default_workers == 1
    assert rkb.lib.rocket_hw_by_name(b"b200") == rkb.lib.rocket_hw_current()
    assert not rkb.lib.rocket_hw_by_name(b"rk3588")


def test_gw_mode_knob(rkb):
    assert rkb.lib.rocket_b200_gw_mode(1) == 0
    assert rkb.lib.rocket_b200_gw_mode(0) == 0
    assert rkb.lib.rocket_b200_gw_mode(-1) == rkb.ROCKET_E_SHAPE
    assert rkb.lib.rocket_activation_name(5) == b"gelu"
    assert rkb.lib.rocket_activation_name(18) == b"log"
    assert rkb.lib.rocket_activation_name(-1) == b"?"
