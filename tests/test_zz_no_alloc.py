"""The allocation-free entry point, called through the C ABI.

fa_forward_noalloc serves callers that may not allocate device memory (for
example a plugin inside a host application that owns all device
allocations): its scratch is one fixed 64 MiB device array instead of a
pool buffer. This test binds libfa_b200.so with ctypes, as such a caller
would, and checks that two calls in a row give the same output as the
regular fa_forward entry point (within the fp16/bf16 tolerance of the
other tests), and that a problem too large for the array is rejected.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np
import pytest

from conftest import ROOT, assert_close_16

LIB = os.path.join(ROOT, "flash_attn_metal_cpp_b200", "libfa_b200.so")


class FaParams(ctypes.Structure):
    _fields_ = [
        ("batch_size", ctypes.c_uint32), ("seqlen_q", ctypes.c_uint32), ("seqlen_k", ctypes.c_uint32),
        ("num_heads_q", ctypes.c_uint32), ("num_heads_k", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
        ("softmax_scale", ctypes.c_float), ("is_causal", ctypes.c_int32), ("window_left", ctypes.c_int32),
        ("window_right", ctypes.c_int32), ("dropout_p", ctypes.c_float), ("has_alibi", ctypes.c_int32),
        ("has_rotary", ctypes.c_int32), ("gqa_group_size", ctypes.c_uint32), ("dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32), ("rope_theta", ctypes.c_float),
        ("q_stride", ctypes.c_int64 * 3), ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3), ("o_stride", ctypes.c_int64 * 3),
        ("alibi_slopes", ctypes.c_void_p),
    ]


def _lib():
    lib = ctypes.CDLL(LIB)
    vp = ctypes.c_void_p
    lib.fa_params_init.argtypes = [ctypes.POINTER(FaParams)]
    lib.fa_forward_noalloc.argtypes = [ctypes.POINTER(FaParams), vp, vp, vp, vp, vp, vp, vp, vp]
    lib.fa_forward_noalloc.restype = ctypes.c_int
    lib.fa_forward.argtypes = [ctypes.POINTER(FaParams), vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_size_t, vp]
    lib.fa_forward.restype = ctypes.c_int
    lib.fa_last_error.restype = ctypes.c_char_p
    lib.fa_init.argtypes = [ctypes.c_int]
    lib.fa_init.restype = ctypes.c_int
    return lib


def _params(lib, B, Sq, Sk, Hq, Hk, D, causal, dtype, out_dtype, theta):
    p = FaParams()
    lib.fa_params_init(ctypes.byref(p))
    p.batch_size, p.seqlen_q, p.seqlen_k = B, Sq, Sk
    p.num_heads_q, p.num_heads_k, p.head_dim = Hq, Hk, D
    p.softmax_scale = 1.0 / math.sqrt(D)
    p.is_causal = int(causal)
    p.dtype, p.out_dtype = dtype, out_dtype
    if theta:
        p.has_rotary, p.rope_theta = 1, theta
    return p


def test_noalloc_rejects_oversized_problem():
    """Runs without a GPU: the size check happens before any device call."""
    lib = _lib()
    p = _params(lib, 8, 8192, 8192, 32, 8, 128, True, 1, 2, 500000.0)  # bf16 + RoPE: ~900 MB of staging
    st = lib.fa_forward_noalloc(ctypes.byref(p), 16, 16, 16, 16, None, None, None, None)
    assert st == 1  # FA_ERR_INVALID_ARG
    assert b"fixed" in lib.fa_last_error() and b"scratch" in lib.fa_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name,theta", [("bfloat16", 500000.0), ("float16", 10000.0), ("bfloat16", None)])
def test_noalloc_matches_fa_forward_twice(cuda_device, dtype_name, theta):
    import torch

    lib = _lib()
    assert lib.fa_init(0) == 0, lib.fa_last_error()
    tdt = {"bfloat16": torch.bfloat16, "float16": torch.float16}[dtype_name]
    code = {"bfloat16": 1, "float16": 0}[dtype_name]
    B, S, Hq, Hk, D = 2, 1500, 8, 2, 128
    g = torch.Generator(device=cuda_device).manual_seed(99)
    q = torch.randn((B, S, Hq, D), generator=g, device=cuda_device).to(tdt)
    k = torch.randn((B, S, Hk, D), generator=g, device=cuda_device).to(tdt)
    v = torch.randn((B, S, Hk, D), generator=g, device=cuda_device).to(tdt)
    p = _params(lib, B, S, S, Hq, Hk, D, True, code, 2, theta)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream

    ref = torch.empty((B, S, Hq, D), dtype=torch.float32, device=cuda_device)
    ref_lse = torch.empty((B, Hq, S), dtype=torch.float32, device=cuda_device)
    st = lib.fa_forward(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(),
                        ref_lse.data_ptr(), None, None, None, 0, stream)
    assert st == 0, lib.fa_last_error()
    for call in range(2):
        out = torch.full((B, S, Hq, D), float("nan"), dtype=torch.float32, device=cuda_device)
        lse = torch.full((B, Hq, S), float("nan"), dtype=torch.float32, device=cuda_device)
        st = lib.fa_forward_noalloc(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                    lse.data_ptr(), None, None, stream)
        assert st == 0, lib.fa_last_error()
        torch.cuda.synchronize()
        assert_close_16(out.cpu().numpy(), ref.cpu().numpy(), f"noalloc call {call}")
        assert np.abs(lse.cpu().numpy() - ref_lse.cpu().numpy()).max() <= 1e-3
