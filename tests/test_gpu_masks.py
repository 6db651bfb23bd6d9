"""Sliding-window and ALiBi masks (common.metal:95-128) on the GPU against the oracle.

The reference declares both (FlashAttentionParams window_left / window_right /
has_alibi, python/bindings.cpp:175-199) but its kernel never applies them, so
the oracle's restatement of common.metal is the pin. Each case runs through
the torch device path and, for one shape, the NumPy host path. Bars: 16-bit
inputs with float32 output max-abs <= 2e-3 and mean-abs <= 2e-4, LSE
max-abs <= 1e-3; fp32 inputs 1e-5 relative.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import assert_close_16, assert_close_32, err_stats
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(shape_q, shape_kv, dtype, seed, amp=1.0):
    import torch

    gen = torch.Generator(device="cpu").manual_seed(seed)
    q = (torch.randn(shape_q, generator=gen) * amp).to(dtype)
    k = (torch.randn(shape_kv, generator=gen) * amp).to(dtype)
    v = (torch.randn(shape_kv, generator=gen) * amp).to(dtype)
    return q, k, v


def _slopes(hq):
    # The usual geometric ALiBi slopes 2^(-8 i / H), i = 1..H.
    return np.array([2.0 ** (-8.0 * (i + 1) / hq) for i in range(hq)], np.float32)


CASES = [
    # B, Sq, Sk, Hq, Hk, D, dtype, causal, window, alibi, theta
    (2, 700, 700, 4, 2, 128, "bfloat16", True, (256, -1), False, 1e4),    # causal + left window (tile skip)
    (1, 1000, 1000, 8, 1, 128, "bfloat16", False, (100, 37), False, None),  # two-sided window
    (1, 513, 513, 4, 4, 64, "float16", False, (-1, 64), False, None),     # right window only
    (2, 600, 600, 4, 2, 128, "float16", True, None, True, None),          # causal ALiBi
    (1, 777, 777, 8, 2, 128, "bfloat16", False, None, True, 5e5),         # non-causal ALiBi + RoPE
    (1, 900, 900, 4, 1, 64, "bfloat16", True, (300, 0), True, 1e4),       # window + ALiBi
    (1, 300, 400, 2, 1, 40, "float32", True, (64, 16), True, None),       # CUDA-core kernel, Sq != Sk
    (1, 256, 256, 4, 4, 96, "float16", False, (32, 32), True, None),      # D = 96 zero-padded to 128 (tensor cores)
]


@pytest.mark.parametrize("B,Sq,Sk,Hq,Hk,D,dtype,causal,window,alibi,theta", CASES)
def test_window_alibi_match_oracle(fa, cuda_device, B, Sq, Sk, Hq, Hk, D, dtype, causal, window, alibi, theta):
    import torch

    tdt = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[dtype]
    q, k, v = _inputs((B, Sq, Hq, D), (B, Sk, Hk, D), tdt, seed=Sq + Hq + D)
    scale = 1 / math.sqrt(D)
    slopes = _slopes(Hq) if alibi else None
    kw = {}
    if window is not None:
        kw["window_size"] = window
    if alibi:
        kw["alibi_slopes"] = torch.from_numpy(slopes)
    if theta:
        kw["rope_theta"] = theta
    out, lse = fa.forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), softmax_scale=scale,
                          is_causal=causal, out_dtype="float32", return_lse=True, **kw)
    torch.cuda.synchronize()
    fa.check_status()
    qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
    okw = dict(causal=causal, softmax_scale=scale, return_lse=True, window=window, alibi_slopes=slopes)
    if theta:
        ref_o, ref_l = orc.attention_with_rope(qn, kn, vn, theta=theta, **okw)
    else:
        ref_o, ref_l = orc.attention_ref(qn, kn, vn, **okw)
    got = out.cpu().numpy()
    if dtype == "float32":
        assert_close_32(got, ref_o, "window/alibi fp32")
    else:
        assert_close_16(got, ref_o, "window/alibi")
    gl = lse.cpu().numpy()
    assert np.array_equal(np.isneginf(gl), np.isneginf(ref_l))
    fin = np.isfinite(ref_l)
    assert np.abs(gl[fin] - ref_l[fin]).max() <= 1e-3


def test_window_alibi_host_path_and_zero_scale(fa, cuda_device):
    """NumPy host path with window + ALiBi (slopes copied from host memory), and
    ALiBi with softmax_scale = 0 (scores are the bias alone)."""
    import torch

    q, k, v = _inputs((2, 640, 4, 128), (2, 640, 2, 128), torch.float16, seed=5)
    qn, kn, vn = (x.numpy() for x in (q, k, v))
    sl = _slopes(4)
    out = fa.forward(qn, kn, vn, softmax_scale=0.09, is_causal=True, alibi_slopes=sl, window_size=(200, -1),
                     out_dtype="float32")
    ref = orc.attention_ref(qn.astype(np.float32), kn.astype(np.float32), vn.astype(np.float32), causal=True,
                            softmax_scale=0.09, window=(200, -1), alibi_slopes=sl)
    assert_close_16(out, ref, "host path window+alibi")
    out0 = fa.forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), softmax_scale=0.0, is_causal=False,
                      alibi_slopes=torch.from_numpy(sl), out_dtype="float32")
    ref0 = orc.attention_ref(qn.astype(np.float32), kn.astype(np.float32), vn.astype(np.float32), causal=False,
                             softmax_scale=0.0, alibi_slopes=sl)
    assert_close_16(out0.cpu().numpy(), ref0, "alibi with zero scale")


def test_window_skips_tiles_at_long_context(fa, cuda_device):
    """A 1024-key causal window over S = 16384 visits ~9 of 128 KV tiles per
    query tile; sampled rows against the oracle."""
    import torch

    q, k, v = _inputs((1, 16384, 8, 128), (1, 16384, 1, 128), torch.bfloat16, seed=6, amp=0.5)
    out = fa.forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), softmax_scale=1 / math.sqrt(128),
                     is_causal=True, window_size=(1024, 0), rope_theta=5e5, out_dtype="float32")
    torch.cuda.synchronize()
    qn, kn, vn = (x.float().numpy() for x in (q[:, :, :2], k, v))
    for r0, r1 in [(0, 128), (5000, 5200), (16256, 16384)]:
        ref = orc.attention_with_rope(qn, kn, vn, True, 1 / math.sqrt(128), theta=5e5, q_range=(r0, r1),
                                      window=(1024, 0))
        mx, mean = err_stats(out[:, r0:r1, :2].cpu().numpy(), ref[:, r0:r1])
        assert mx <= 2e-3 and mean <= 2e-4, (r0, mx, mean)
