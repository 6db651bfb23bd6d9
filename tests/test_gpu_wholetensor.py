"""Whole-tensor parity at the full configuration sizes.

The CPU oracle is too slow to evaluate every element of the long
configurations, so every element of O and LSE is compared against
gpu_reference.attention_fp32: the oracle's formula (test.py:39-93 plus
rotate-half RoPE, common.metal:150-167) evaluated with fp32 matmuls on the
GPU, chunked per (batch, KV head) and query-row block. That evaluation is
first checked against the NumPy oracle on slices of the same inputs, then
trusted for the whole output -- which covers every CTA's (block, head,
batch) placement, the heaviest-first launch order and, for cfg4, the host
path's chunking, where sampled rows could miss a misplaced tile (the
reference's own check compares every element, test.py:96-123).

Bars (fp16/bf16 inputs, float32 output): max-abs <= 2e-3, mean-abs <= 2e-4;
LSE max-abs <= 1e-3.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import TOL_MAX_ABS_16, TOL_MEAN_ABS_16
from gpu_reference import attention_fp32, compare_whole, oracle_slice

pytestmark = pytest.mark.gpu

# name: (B, S, Hq, Hkv, D, dtype, theta, amplitude, oracle slices [(b, h, (r0, r1))])
CONFIGS = {
    "cfg3_fp16_causal_rope_B8_S2048_H32": (8, 2048, 32, 32, 128, "float16", 1e4, 1.0,
                                          [(0, 0, (0, 256)), (7, 31, (1792, 2048))]),
    "cfg4_bf16_gqa_causal_rope_B4_S8192_Hq32_Hkv8": (4, 8192, 32, 8, 128, "bfloat16", 5e5, 1.0,
                                                    [(0, 0, (0, 128)), (3, 30, (8064, 8192))]),
    "cfg5a_bf16_gqa_causal_rope_B1_S65536_Hq64_Hkv8": (1, 65536, 64, 8, 128, "bfloat16", 5e5, 0.5,
                                                      [(0, 0, (0, 128)), (0, 63, (65408, 65536))]),
}


def _inputs(B, S, Hq, Hkv, D, dtype, amp, seed, device):
    import torch

    tdt = {"float16": torch.float16, "bfloat16": torch.bfloat16}[dtype]
    g = torch.Generator(device=device).manual_seed(seed)
    q = (torch.randn((B, S, Hq, D), generator=g, device=device) * amp).to(tdt)
    k = (torch.randn((B, S, Hkv, D), generator=g, device=device) * amp).to(tdt)
    v = (torch.randn((B, S, Hkv, D), generator=g, device=device) * amp).to(tdt)
    return q, k, v


def _validated_reference(q, k, v, scale, theta, slices, row_block):
    """GPU fp32 reference of the whole problem, after checking it against the
    NumPy oracle on the given slices (it must agree to fp32 rounding)."""
    ref_o, ref_l = attention_fp32(q, k, v, True, scale, theta, row_block=row_block)
    for b, h, rows in slices:
        o_np, l_np = oracle_slice(q, k, v, True, scale, theta, b, h, rows)
        d_o = np.abs(ref_o[b, rows[0]:rows[1], h].cpu().numpy() - o_np).max()
        d_l = np.abs(ref_l[b, h, rows[0]:rows[1]].cpu().numpy() - l_np).max()
        assert d_o <= 2e-5 and d_l <= 2e-5, f"GPU reference disagrees with the oracle: O {d_o:.2e}, LSE {d_l:.2e}"
    return ref_o, ref_l


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_whole_output_matches_reference(fa, cuda_device, name):
    import torch

    B, S, Hq, Hkv, D, dtype, theta, amp, slices = CONFIGS[name]
    q, k, v = _inputs(B, S, Hq, Hkv, D, dtype, amp, seed=40 + sorted(CONFIGS).index(name), device=cuda_device)
    scale = 1 / math.sqrt(D)
    out, lse = fa.forward(q, k, v, softmax_scale=scale, is_causal=True, out_dtype="float32", rope_theta=theta,
                          return_lse=True)
    torch.cuda.synchronize()
    fa.check_status()
    ref_o, ref_l = _validated_reference(q, k, v, scale, theta, slices, row_block=2048 if S > 8192 else 4096)
    mx, mean = compare_whole(out, ref_o, TOL_MAX_ABS_16, TOL_MEAN_ABS_16, name)
    lmx = float((lse - ref_l).abs().max())
    assert lmx <= 1e-3, f"{name}: LSE max_abs={lmx:.3e}"
    print(f"{name}: every element of O: max_abs {mx:.2e} mean_abs {mean:.2e}; LSE max_abs {lmx:.2e}")
    if name.startswith("cfg4"):
        # The host-pointer path (chunked over batches and query-row blocks,
        # heaviest block first) on the same inputs: bit-identical output.
        qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
        out_h, lse_h = fa.forward(qh, kh, vh, softmax_scale=scale, is_causal=True, out_dtype="float32",
                                  rope_theta=theta, return_lse=True)
        assert torch.equal(out_h, out.cpu()) and torch.equal(lse_h, lse.cpu())
