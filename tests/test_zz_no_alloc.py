"""The allocation-free entry point, called through the C ABI.

fa_forward_noalloc serves callers that may not allocate device memory (for
example a plugin inside a host application that owns all device
allocations): its scratch is one fixed 64 MiB device array instead of a
pool buffer. These tests bind libfa_b200.so with ctypes, as such a caller
would, and check that calls in a row give the same output as the regular
fa_forward entry point (within the fp16/bf16 tolerance of the other tests)
for every kind of scratch use: none (fp16 without RoPE), fp16 staging of
bf16 and rotated operands, RoPE tables from theta or from the caller,
zero-padded operands of other head dims, and a small call after a larger
one (every byte a call reads from the shared array is written earlier in
the same call). Warm calls must leave the device's free memory unchanged,
and a problem too large for the array is rejected.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import assert_close_16
from fa_ctypes import FA_BF16, FA_F16, FA_F32, load_lib, make_params
from oracle import attention_oracle as orc


def test_noalloc_rejects_oversized_problem():
    """Runs without a GPU: the size check happens before any device call."""
    lib = load_lib()
    p = make_params(lib, 8, 8192, 8192, 32, 8, 128, True, FA_BF16, FA_F32, 500000.0)  # ~900 MB of staging
    st = lib.fa_forward_noalloc(ctypes.byref(p), 16, 16, 16, 16, None, None, None, None)
    assert st == 1  # FA_ERR_INVALID_ARG
    assert b"fixed" in lib.fa_last_error() and b"scratch" in lib.fa_last_error()


def _inputs(cuda_device, B, S, Hq, Hk, D, tdt, seed):
    import torch

    g = torch.Generator(device=cuda_device).manual_seed(seed)
    q = torch.randn((B, S, Hq, D), generator=g, device=cuda_device).to(tdt)
    k = torch.randn((B, S, Hk, D), generator=g, device=cuda_device).to(tdt)
    v = torch.randn((B, S, Hk, D), generator=g, device=cuda_device).to(tdt)
    return q, k, v


def _run_both(lib, cuda_device, B, S, Hq, Hk, D, dtype_name, theta, tables=False, calls=2, seed=99):
    """fa_forward once, then fa_forward_noalloc `calls` times; each noalloc
    output must match fa_forward's. Returns the noalloc outputs."""
    import torch

    tdt = {"bfloat16": torch.bfloat16, "float16": torch.float16}[dtype_name]
    code = {"bfloat16": FA_BF16, "float16": FA_F16}[dtype_name]
    q, k, v = _inputs(cuda_device, B, S, Hq, Hk, D, tdt, seed)
    p = make_params(lib, B, S, S, Hq, Hk, D, True, code, FA_F32, theta)
    cs = sn = None
    if tables:
        c_np, s_np = orc.rope_tables(S, D, theta)
        cs, sn = torch.from_numpy(c_np).to(cuda_device), torch.from_numpy(s_np).to(cuda_device)
        p.has_rotary, p.rope_theta = 1, 0.0  # tables only
    cp = cs.data_ptr() if cs is not None else None
    sp = sn.data_ptr() if sn is not None else None
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    ref = torch.empty((B, S, Hq, D), dtype=torch.float32, device=cuda_device)
    ref_lse = torch.empty((B, Hq, S), dtype=torch.float32, device=cuda_device)
    st = lib.fa_forward(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(),
                        ref_lse.data_ptr(), cp, sp, None, 0, stream)
    assert st == 0, lib.fa_last_error()
    outs = []
    for call in range(calls):
        out = torch.full((B, S, Hq, D), float("nan"), dtype=torch.float32, device=cuda_device)
        lse = torch.full((B, Hq, S), float("nan"), dtype=torch.float32, device=cuda_device)
        st = lib.fa_forward_noalloc(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                    lse.data_ptr(), cp, sp, stream)
        assert st == 0, lib.fa_last_error()
        torch.cuda.synchronize()
        assert lib.fa_noalloc_check_status() == 0, lib.fa_last_error()
        assert_close_16(out.cpu().numpy(), ref.cpu().numpy(), f"noalloc D{D} {dtype_name} call {call}")
        assert np.abs(lse.cpu().numpy() - ref_lse.cpu().numpy()).max() <= 1e-3
        outs.append(out)
    return outs


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name,theta", [("bfloat16", 500000.0), ("float16", 10000.0), ("bfloat16", None),
                                              ("float16", None)])
def test_noalloc_matches_fa_forward_twice(cuda_device, dtype_name, theta):
    """bf16 / fp16, with RoPE from theta (tables in the array), and fp16
    without RoPE (no scratch at all)."""
    lib = load_lib()
    assert lib.fa_init(0) == 0, lib.fa_last_error()
    _run_both(lib, cuda_device, 2, 1500, 8, 2, 128, dtype_name, theta)


@pytest.mark.gpu
def test_noalloc_with_caller_tables(cuda_device):
    """RoPE from the caller's cos/sin tables (device memory the caller owns)."""
    lib = load_lib()
    assert lib.fa_init(0) == 0, lib.fa_last_error()
    _run_both(lib, cuda_device, 1, 777, 4, 1, 128, "bfloat16", 10000.0, tables=True)


@pytest.mark.gpu
@pytest.mark.parametrize("D,dtype_name,theta", [(96, "bfloat16", 10000.0), (40, "float16", None)])
def test_noalloc_other_head_dims(cuda_device, D, dtype_name, theta):
    """Head dims other than 64 / 128 run zero-padded on the tensor cores,
    the padded operands and output living in the array."""
    lib = load_lib()
    assert lib.fa_init(0) == 0, lib.fa_last_error()
    _run_both(lib, cuda_device, 2, 600, 4, 2, D, dtype_name, theta)


@pytest.mark.gpu
def test_noalloc_small_call_after_large_one(cuda_device):
    """A large call fills most of the array; a smaller call with another
    shape then reads only what it wrote itself."""
    lib = load_lib()
    assert lib.fa_init(0) == 0, lib.fa_last_error()
    _run_both(lib, cuda_device, 2, 4000, 8, 2, 128, "bfloat16", 500000.0, calls=1, seed=1)
    _run_both(lib, cuda_device, 1, 300, 2, 1, 128, "bfloat16", 10000.0, calls=1, seed=2)
    _run_both(lib, cuda_device, 1, 450, 4, 4, 64, "float16", 10000.0, calls=1, seed=3)


@pytest.mark.gpu
def test_noalloc_leaves_free_memory_unchanged(cuda_device):
    """Warm calls allocate nothing: the device's free memory is the same
    before and after several calls of every scratch kind."""
    import torch

    lib = load_lib()
    assert lib.fa_init(0) == 0, lib.fa_last_error()
    cases = [(1, 1000, 8, 2, 128, torch.bfloat16, FA_BF16, 500000.0), (1, 500, 4, 2, 96, torch.float16, FA_F16, 1e4),
             (1, 800, 4, 4, 64, torch.float16, FA_F16, None)]
    bufs = []
    for (B, S, Hq, Hk, D, tdt, code, theta) in cases:
        q, k, v = _inputs(cuda_device, B, S, Hq, Hk, D, tdt, 7)
        out = torch.empty((B, S, Hq, D), dtype=torch.float32, device=cuda_device)
        lse = torch.empty((B, Hq, S), dtype=torch.float32, device=cuda_device)
        bufs.append((make_params(lib, B, S, S, Hq, Hk, D, True, code, FA_F32, theta), q, k, v, out, lse))
    stream = torch.cuda.current_stream(cuda_device).cuda_stream

    def call_all():
        for p, q, k, v, out, lse in bufs:
            st = lib.fa_forward_noalloc(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        lse.data_ptr(), None, None, stream)
            assert st == 0, lib.fa_last_error()
        torch.cuda.synchronize()

    call_all()  # first calls: symbol lookup and lazy loading of the kernels
    free0, _ = torch.cuda.mem_get_info(cuda_device)
    for _ in range(3):
        call_all()
    free1, _ = torch.cuda.mem_get_info(cuda_device)
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes across warm calls"
    assert lib.fa_noalloc_check_status() == 0
