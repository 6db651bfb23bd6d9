"""Failure detection on the GPU without a fault (the reference reports errors
as RuntimeError, python/bindings.cpp:224-232).

Every in-kernel wait of the tensor-core kernel is bounded. Here a test hook
(fa_test_stall_next_launch) makes one CTA's K producer withhold one K tile,
so the waits for it run out after a 1 ms limit: the kernel records a
timeout in its status word, releases its tensor memory and returns. The
host must then see FA_ERR_TIMEOUT (RuntimeError through the module), and
the next normal call on the same context must be correct. Nothing here
traps, faults or hangs the GPU: the longest wait is the 1 ms limit.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

from conftest import assert_close_16
from fa_ctypes import FA_ERR_TIMEOUT, FA_F16, FA_F32, load_lib, make_params
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

B, S, H, D = 1, 1024, 2, 128  # causal: the first CTA (heaviest block) has 8 K tiles


def _inputs(cuda_device):
    import torch

    g = torch.Generator(device=cuda_device).manual_seed(77)
    return tuple(torch.randn((B, S, H, D), generator=g, device=cuda_device).to(torch.float16) for _ in range(3))


def _oracle(q, k, v):
    return orc.attention_ref(*(x.float().cpu().numpy() for x in (q, k, v)), causal=True,
                             softmax_scale=1 / math.sqrt(D))


@pytest.mark.parametrize("noalloc", [False, True])
def test_wait_timeout_reported_and_next_call_correct(cuda_device, noalloc):
    import torch

    lib = load_lib()
    assert lib.fa_init(0) == 0, lib.fa_last_error()
    q, k, v = _inputs(cuda_device)
    p = make_params(lib, B, S, S, H, H, D, True, FA_F16, FA_F32)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    check = lib.fa_noalloc_check_status if noalloc else lib.fa_check_device_status

    def call(out):
        if noalloc:
            return lib.fa_forward_noalloc(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                          None, None, None, stream)
        return lib.fa_forward(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), None,
                              None, None, None, 0, stream)

    assert lib.fa_check_device_status() == 0 and lib.fa_noalloc_check_status() == 0
    limit0 = lib.fa_get_wait_limit()
    out = torch.zeros((B, S, H, D), dtype=torch.float32, device=cuda_device)
    assert lib.fa_set_wait_limit(1e-3) == 0
    try:
        assert lib.fa_test_stall_next_launch(1) == 0
        assert call(out) == 0, lib.fa_last_error()
        torch.cuda.synchronize()  # returns: the stalled CTA gave up its waits
    finally:
        assert lib.fa_set_wait_limit(limit0) == 0
    assert check() == FA_ERR_TIMEOUT
    assert b"time limit" in lib.fa_last_error()
    assert check() == 0, "the status word is cleared by reading it"
    # The context is intact: the same call now completes and matches the oracle.
    out2 = torch.full((B, S, H, D), float("nan"), dtype=torch.float32, device=cuda_device)
    assert call(out2) == 0, lib.fa_last_error()
    torch.cuda.synchronize()
    assert check() == 0
    assert_close_16(out2.cpu().numpy(), _oracle(q, k, v), "call after a timeout")


def test_timeout_raises_through_the_module(fa, cuda_device):
    """The module surface turns the recorded timeout into RuntimeError."""
    import torch

    lib = load_lib()
    q, k, v = _inputs(cuda_device)
    limit0 = lib.fa_get_wait_limit()
    assert lib.fa_set_wait_limit(1e-3) == 0
    try:
        assert lib.fa_test_stall_next_launch(2) == 0  # armed for this thread's next tensor-core launch
        fa.forward(q, k, v, softmax_scale=1 / math.sqrt(D), is_causal=True)
        torch.cuda.synchronize()
    finally:
        assert lib.fa_set_wait_limit(limit0) == 0
    with pytest.raises(RuntimeError, match="time limit"):
        fa.check_status()
    fa.check_status()  # cleared
    out = fa.forward(q, k, v, softmax_scale=1 / math.sqrt(D), is_causal=True, out_dtype="float32")
    torch.cuda.synchronize()
    fa.check_status()
    assert_close_16(out.cpu().numpy(), _oracle(q, k, v), "module call after a timeout")
    # The host-pointer path checks the status itself and raises.
    assert lib.fa_set_wait_limit(1e-3) == 0
    try:
        assert lib.fa_test_stall_next_launch(1) == 0
        with pytest.raises(RuntimeError, match="Forward pass error: .*time limit"):
            fa.forward(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), softmax_scale=1 / math.sqrt(D),
                       is_causal=True)
    finally:
        assert lib.fa_set_wait_limit(limit0) == 0
    np.testing.assert_array_equal(
        fa.forward(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), softmax_scale=1 / math.sqrt(D),
                   is_causal=True), out.cpu().numpy().astype(np.float16))
