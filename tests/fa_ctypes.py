"""ctypes binding of the C ABI (include/fa_b200.h) shared by the tests that
call libfa_b200.so directly, the way a non-Python host binds it: the
fa_params mirror, the library loader with argument types, and a helper
that fills fa_params for a contiguous problem. tests/test_params_layout.py
checks this mirror against the header's C layout."""
from __future__ import annotations

import ctypes
import math
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(ROOT, "flash_attn_metal_cpp_b200", "libfa_b200.so")

# fa_status codes
FA_OK, FA_ERR_INVALID_ARG, FA_ERR_UNSUPPORTED, FA_ERR_CUDA, FA_ERR_TIMEOUT = 0, 1, 2, 3, 4
# fa_dtype codes
FA_F16, FA_BF16, FA_F32 = 0, 1, 2


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


def load_lib():
    lib = ctypes.CDLL(LIB_PATH)
    vp, P = ctypes.c_void_p, ctypes.POINTER(FaParams)
    sigs = {
        "fa_params_init": ([P], None),
        "fa_init": ([ctypes.c_int], ctypes.c_int),
        "fa_forward": ([P, vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_size_t, vp], ctypes.c_int),
        "fa_forward_noalloc": ([P, vp, vp, vp, vp, vp, vp, vp, vp], ctypes.c_int),
        "fa_noalloc_check_status": ([], ctypes.c_int),
        "fa_check_device_status": ([], ctypes.c_int),
        "fa_set_wait_limit": ([ctypes.c_double], ctypes.c_int),
        "fa_get_wait_limit": ([], ctypes.c_double),
        "fa_test_stall_next_launch": ([ctypes.c_int32], ctypes.c_int),
        "fa_workspace_size": ([P], ctypes.c_size_t),
        "fa_tensor_bytes": ([ctypes.c_uint32] * 4 + [ctypes.c_int32], ctypes.c_size_t),
        "fa_pool_clear": ([], ctypes.c_int),
        "fa_last_error": ([], ctypes.c_char_p),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


def make_params(lib, B, Sq, Sk, Hq, Hk, D, causal, dtype, out_dtype=-1, theta=None, scale=None) -> FaParams:
    p = FaParams()
    lib.fa_params_init(ctypes.byref(p))
    p.batch_size, p.seqlen_q, p.seqlen_k = B, Sq, Sk
    p.num_heads_q, p.num_heads_k, p.head_dim = Hq, Hk, D
    p.softmax_scale = 1.0 / math.sqrt(D) if scale is None else scale
    p.is_causal = int(causal)
    p.dtype, p.out_dtype = dtype, out_dtype
    if theta:
        p.has_rotary, p.rope_theta = 1, theta
    return p
