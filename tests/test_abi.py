"""The C-ABI library loads and exports every symbol include/fa_b200.h declares;
host-only entry points behave as documented (CPU, no compute calls)."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

from conftest import ROOT
from oracle import attention_oracle as orc
from fa_ctypes import FaParams

LIB = os.path.join(ROOT, "flash_attn_metal_cpp_b200", "libfa_b200.so")
HEADER = os.path.join(ROOT, "include", "fa_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fa_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    names = _declared()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_params_defaults_and_sizes():
    lib = ctypes.CDLL(LIB)
    lib.fa_params_init.argtypes = [ctypes.POINTER(FaParams)]
    p = FaParams()
    p.head_dim = 99
    lib.fa_params_init(ctypes.byref(p))
    assert p.head_dim == 0 and p.window_left == -1 and p.window_right == -1 and p.out_dtype == -1
    assert p.softmax_scale == 0.0 and p.dtype == 0
    lib.fa_tensor_bytes.restype = ctypes.c_size_t
    lib.fa_tensor_bytes.argtypes = [ctypes.c_uint32] * 4 + [ctypes.c_int32]
    assert lib.fa_tensor_bytes(2, 3, 4, 64, 1) == 2 * 3 * 4 * 64 * 2
    assert lib.fa_tensor_bytes(2, 3, 4, 64, 2) == 2 * 3 * 4 * 64 * 4


def test_workspace_size_per_path():
    lib = ctypes.CDLL(LIB)
    lib.fa_params_init.argtypes = [ctypes.POINTER(FaParams)]
    lib.fa_workspace_size.argtypes = [ctypes.POINTER(FaParams)]
    lib.fa_workspace_size.restype = ctypes.c_size_t

    def ws(dtype, rope, D=128):
        p = FaParams()
        lib.fa_params_init(ctypes.byref(p))
        p.batch_size, p.seqlen_q, p.seqlen_k, p.num_heads_q, p.num_heads_k, p.head_dim = 2, 1000, 1000, 8, 2, D
        p.dtype, p.has_rotary, p.rope_theta = dtype, int(rope), 1e4
        return lib.fa_workspace_size(ctypes.byref(p))

    q16 = 2 * 1000 * 8 * 128 * 2
    kv16 = 2 * 1000 * 2 * 128 * 2
    rec = 256                                     # staging record (per-tensor range exponents)
    assert ws(0, False) == 0                      # fp16, no RoPE: zero-copy
    assert ws(1, False) == rec + kv16             # bf16: V staged as fp16
    assert ws(0, True) == rec + q16 + kv16        # fp16 + RoPE: rotated Q, K
    assert ws(1, True) == rec + q16 + 2 * kv16    # bf16 + RoPE: Q, K, V
    assert ws(2, True) == 0                       # fp32: CUDA-core kernel, RoPE on load
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    q128, kv128 = 2 * 1000 * 8 * 128 * 2, 2 * 1000 * 2 * 128 * 2
    assert ws(0, True, D=96) == rec + up(q128) + 2 * up(kv128) + up(q128)  # padded to 128: Q, K, V and O
    assert ws(1, False, D=40) == rec + up(q128 // 2) + 2 * up(kv128 // 2) + up(q128 // 2)  # padded to 64
    assert ws(0, True, D=160) == 0                # head dims above 128: CUDA-core kernel


def test_wait_limit_setting():
    """The in-kernel wait limit is a host setting (no device needed)."""
    from fa_ctypes import load_lib

    lib = load_lib()
    assert abs(lib.fa_get_wait_limit() - 2.0) < 1e-12 or lib.fa_get_wait_limit() > 0
    before = lib.fa_get_wait_limit()
    try:
        assert lib.fa_set_wait_limit(0.5) == 0
        assert abs(lib.fa_get_wait_limit() - 0.5) < 1e-9
        assert lib.fa_set_wait_limit(0.0) == 1 and b"wait limit" in lib.fa_last_error()
        assert lib.fa_set_wait_limit(-1.0) == 1
        assert lib.fa_set_wait_limit(float("nan")) == 1
        assert abs(lib.fa_get_wait_limit() - 0.5) < 1e-9  # rejected values leave it unchanged
        assert lib.fa_test_stall_next_launch(-1) == 1
    finally:
        lib.fa_set_wait_limit(before)


def test_rope_tables_match_oracle():
    lib = ctypes.CDLL(LIB)
    lib.fa_rope_tables.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_float]
    cs = np.zeros((300, 64), np.float32)
    sn = np.zeros((300, 64), np.float32)
    assert lib.fa_rope_tables(cs.ctypes.data, sn.ctypes.data, 300, 128, ctypes.c_float(500000.0)) == 0
    c_ref, s_ref = orc.rope_tables(300, 128, 500000.0)
    np.testing.assert_array_equal(cs, c_ref)
    np.testing.assert_array_equal(sn, s_ref)


def test_errors_without_a_device():
    lib = ctypes.CDLL(LIB)
    lib.fa_init.argtypes = [ctypes.c_int]
    lib.fa_last_error.restype = ctypes.c_char_p
    import torch

    if torch.cuda.is_available():
        return
    assert lib.fa_init(0) == 7  # FA_ERR_NO_DEVICE
    assert lib.fa_last_error()
    # argument validation happens before any device call
    lib.fa_params_init.argtypes = [ctypes.POINTER(FaParams)]
    p = FaParams()
    lib.fa_params_init(ctypes.byref(p))
    p.batch_size = p.seqlen_q = p.seqlen_k = p.num_heads_q = p.num_heads_k = 1
    p.head_dim = 64
    p.dropout_p = 0.1
    lib.fa_forward_host.argtypes = [ctypes.POINTER(FaParams)] + [ctypes.c_void_p] * 7
    assert lib.fa_forward_host(ctypes.byref(p), 1, 1, 1, 1, None, None, None) == 2  # UNSUPPORTED
    assert b"dropout" in lib.fa_last_error()
    p.dropout_p = 0.0
    p.num_heads_q, p.num_heads_k = 3, 2
    assert lib.fa_forward_host(ctypes.byref(p), 1, 1, 1, 1, None, None, None) == 1  # INVALID_ARG
