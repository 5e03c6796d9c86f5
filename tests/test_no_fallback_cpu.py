"""CPU: the library has no host fallback.  Without a device handle every
compute entry returns an error and leaves its output untouched; argument
validation (shapes, policies) answers without a device."""
import ctypes

import numpy as np


def P(a):
    return ctypes.c_void_p(a.ctypes.data)


def test_matmuls_fail_loudly_without_a_device(rkb):
    L = rkb.lib
    A = np.ones((64, 512), np.int8)
    B = np.ones((256, 512), np.int8)
    C = np.full((64, 256), 7, np.int32)
    assert L.rocket_matmul_int8(-1, 64, 512, 256, P(A), P(B), P(C)) != 0
    assert (C == 7).all()
    A16 = np.ones((64, 512), np.float16)
    B16 = np.ones((256, 512), np.float16)
    C16 = np.full((64, 256), 3, np.float16)
    assert L.rocket_matmul_fp16(-1, 64, 512, 256, P(A16), P(B16), P(C16)) != 0
    assert (C16 == 3).all()


def test_encoder_ops_fail_loudly_without_a_device(rkb):
    L = rkb.lib
    x = np.ones((8, 64), np.float16)
    g = np.ones(64, np.float16)
    y = np.full((8, 64), 5, np.float16)
    assert L.rocket_layernorm_fp16(-1, 8, 64, P(x), P(g), P(g), ctypes.c_float(1e-5), P(y)) != 0
    assert (y == 5).all()
    loss = np.full(8, 9, np.float32)
    t = np.zeros(8, np.int32)
    assert L.rocket_cross_entropy_fp16(-1, 8, 64, P(x), P(t), P(loss)) != 0
    assert (loss == 9).all()


def test_shape_validation_needs_no_device(rkb):
    L = rkb.lib
    E_SHAPE = rkb.ROCKET_E_SHAPE
    x = np.ones(16, np.float16)
    o = np.zeros(16, np.float32)
    assert L.rocket_reduce_feature_fp16(-1, 0, 16, P(x), P(o), 0) == E_SHAPE
    assert L.rocket_cumsum_fp16(-1, 4, 0, P(x), P(x), 0, 0) == E_SHAPE
    # flash attention: n_head not a multiple of n_kv_heads; head_dim not a multiple of 32
    q = np.zeros(1024, np.float16)
    assert L.rocket_flash_attn_fp16(-1, 8, 8, 64, 64, 3, 2, 0.1, 0.0, P(q), P(q), P(q), None, P(q)) == E_SHAPE
    assert L.rocket_flash_attn_fp16(-1, 8, 8, 40, 64, 2, 2, 0.1, 0.0, P(q), P(q), P(q), None, P(q)) == E_SHAPE
    # int16 exact: K % 32
    a = np.zeros(64, np.int16)
    c = np.zeros(64, np.int64)
    assert L.rocket_matmul_int16_exact(-1, 4, 16, 32, P(a), P(a), P(c)) == E_SHAPE


def test_gemm_policy_validation_needs_no_device(rkb):
    L = rkb.lib
    assert L.rocket_b200_gemm_policy(320, -1) != 0
    assert L.rocket_b200_gemm_policy(0, 2) != 0
    for v in (0, 128, 256, 384, 512):
        assert L.rocket_b200_gemm_policy(v, -1) == 0
    assert L.rocket_b200_gemm_policy(0, -1) == 0
