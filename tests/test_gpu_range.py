"""Inputs beyond the fp16 range on the tensor-core path.

The tensor-core kernel multiplies fp16 operands: bf16 V (and rotated Q/K)
are staged as fp16. A staged tensor whose largest magnitude exceeds 65504
is stored as x * 2^-e with the smallest such power of two, and the kernel
multiplies the scores (Q, K) or O (V) back by 2^e, so inputs anywhere in
the bf16 range (the dtype contract of the path, python/bindings.cpp:136-138,
extended to bf16) give the oracle's result instead of inf.

Tolerance: the fp16/bf16 bar (max-abs 2e-3, mean-abs 2e-4 for N(0,1)
data) scaled by the output's magnitude (max |V|). The softmax scale is
chosen so the logits stay O(1): with saturated logits the output is decided
by near-ties between keys, where any two fp32 evaluations may differ.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _make(cuda_device, B, S, Hq, Hk, D, dtype, q_amp, v_amp, seed):
    import torch

    tdt = {"bfloat16": torch.bfloat16, "float16": torch.float16}[dtype]
    g = torch.Generator(device=cuda_device).manual_seed(seed)
    q = (torch.randn((B, S, Hq, D), generator=g, device=cuda_device) * q_amp)
    k = (torch.randn((B, S, Hk, D), generator=g, device=cuda_device) * q_amp)
    v = (torch.randn((B, S, Hk, D), generator=g, device=cuda_device) * v_amp)
    if dtype == "float16":
        q, k, v = (x.clamp(-65504, 65504) for x in (q, k, v))
    return q.to(tdt), k.to(tdt), v.to(tdt)


def _check(out, q, k, v, scale, theta, what):
    qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
    v_scale = max(1.0, float(np.abs(vn).max()))
    if theta:
        ref = orc.attention_with_rope(qn, kn, vn, True, scale, theta=theta)
    else:
        ref = orc.attention_ref(qn, kn, vn, causal=True, softmax_scale=scale)
    got = np.asarray(out, dtype=np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    d = np.abs(got - ref)
    assert d.max() <= 2e-3 * v_scale and d.mean() <= 2e-4 * v_scale, \
        f"{what}: max_abs={d.max():.3e} mean_abs={d.mean():.3e} (scale {v_scale:.1e})"


@pytest.mark.parametrize("D", [128, 96])
@pytest.mark.parametrize("theta", [None, 10000.0])
def test_bf16_beyond_fp16_range(fa, cuda_device, D, theta):
    """bf16 V at ~1e6 and Q/K at ~1e5 (rotated up to ~5e5): every staged
    tensor overflows fp16 without the rescale."""
    import torch

    q, k, v = _make(cuda_device, 1, 700, 4, 2, D, "bfloat16", 1e5, 1e6, seed=D)
    scale = 1 / (math.sqrt(D) * 1e10)  # logits O(1)
    out = fa.forward(q, k, v, softmax_scale=scale, is_causal=True, out_dtype="float32", rope_theta=theta)
    torch.cuda.synchronize()
    fa.check_status()
    _check(out.cpu().numpy(), q, k, v, scale, theta, f"bf16 D{D} theta {theta}")
    # The same inputs through the host-pointer path (NumPy bfloat16 arrays).
    import ml_dtypes

    qn, kn, vn = (x.float().cpu().numpy().astype(ml_dtypes.bfloat16) for x in (q, k, v))
    out_h = fa.forward(qn, kn, vn, softmax_scale=scale, is_causal=True, out_dtype="float32", rope_theta=theta)
    assert np.array_equal(out_h, out.cpu().numpy())


def test_only_v_beyond_range_and_standard_scale(fa, cuda_device):
    """bf16 V at ~1e6 with Q/K ~N(0,1) and the usual 1/sqrt(D) scale (no
    RoPE: Q K^T runs on the exact bf16 inputs, only V is staged)."""
    import torch

    q, k, v = _make(cuda_device, 2, 500, 8, 2, 128, "bfloat16", 1.0, 1e6, seed=3)
    out = fa.forward(q, k, v, softmax_scale=1 / math.sqrt(128), is_causal=True, out_dtype="float32")
    torch.cuda.synchronize()
    fa.check_status()
    _check(out.cpu().numpy(), q, k, v, 1 / math.sqrt(128), None, "bf16 V 1e6")


def test_fp16_rotation_overflow(fa, cuda_device):
    """fp16 Q/K near the top of the fp16 range: the rotation alone can exceed
    65504 (|x cos - y sin| <= sqrt(2) max)."""
    import torch

    q, k, v = _make(cuda_device, 1, 600, 2, 2, 128, "float16", 4e4, 1.0, seed=4)
    scale = 1 / (math.sqrt(128) * 1.6e9)
    out = fa.forward(q, k, v, softmax_scale=scale, is_causal=True, out_dtype="float32", rope_theta=10000.0)
    torch.cuda.synchronize()
    fa.check_status()
    _check(out.cpu().numpy(), q, k, v, scale, 10000.0, "fp16 rotation overflow")


def test_normal_call_after_rescaled_call(fa, cuda_device):
    """The staging record is cleared after a rescaled call: a following call
    on ordinary inputs (same stream, same workspace) is exact again."""
    import torch

    qb, kb, vb = _make(cuda_device, 1, 640, 4, 2, 128, "bfloat16", 1e5, 1e6, seed=5)
    fa.forward(qb, kb, vb, softmax_scale=1e-11, is_causal=True, rope_theta=5e5)
    q, k, v = _make(cuda_device, 1, 640, 4, 2, 128, "bfloat16", 1.0, 1.0, seed=6)
    a = fa.forward(q, k, v, softmax_scale=0.088, is_causal=True, rope_theta=5e5, out_dtype="float32")
    fa.forward(qb, kb, vb, softmax_scale=1e-11, is_causal=True, rope_theta=5e5)
    b = fa.forward(q, k, v, softmax_scale=0.088, is_causal=True, rope_theta=5e5, out_dtype="float32")
    side = torch.cuda.Stream(cuda_device)  # a fresh per-stream workspace
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(side):
        c = fa.forward(q, k, v, softmax_scale=0.088, is_causal=True, rope_theta=5e5, out_dtype="float32")
    torch.cuda.synchronize()
    fa.check_status()
    assert torch.equal(a, b) and torch.equal(a, c)
    _check(a.cpu().numpy(), q, k, v, 0.088, 5e5, "ordinary call after a rescaled one")


@pytest.mark.parametrize("D", [128, 64])
def test_q_rows_mixed_range(fa, cuda_device, D):
    """A few query rows far beyond the fp16 range among ordinary ones (first,
    second and ragged last query tile, several heads of a GQA group): the
    whole staged Q takes their exponent, and the ordinary rows, scaled down
    with it, still match the oracle. The cos/sin tables come from a view that
    starts 4 bytes off a 16-byte boundary (the staging pass reads table rows
    with 16-byte loads only when the tables are 16-byte aligned)."""
    import torch

    B, S, Hq, Hk, theta = 2, 777, 8, 2, 5e5
    g = torch.Generator(device=cuda_device).manual_seed(40 + D)
    q = torch.randn((B, S, Hq, D), generator=g, device=cuda_device)
    k = torch.randn((B, S, Hk, D), generator=g, device=cuda_device)
    v = torch.randn((B, S, Hk, D), generator=g, device=cuda_device)
    for b, s, h in [(0, 0, 0), (0, 127, 3), (1, 128, 7), (1, 300, 1), (0, 776, 5)]:
        q[b, s, h] *= 1e6
    q, k, v = (x.to(torch.bfloat16) for x in (q, k, v))
    cs, sn = orc.rope_tables(S, D, theta)
    views = []
    for t in (cs, sn):
        base = torch.zeros(t.size + 1, device=cuda_device)
        view = base[1:].view(t.shape)
        view.copy_(torch.from_numpy(t))
        assert view.data_ptr() % 16 != 0
        views.append(view)
    scale = 1 / math.sqrt(D)
    out = fa.forward(q, k, v, softmax_scale=scale, is_causal=True, out_dtype="float32", cos=views[0], sin=views[1])
    torch.cuda.synchronize()
    fa.check_status()
    _check(out.cpu().numpy(), q, k, v, scale, theta, f"bf16 D{D} mixed Q rows")
