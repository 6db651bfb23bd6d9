"""PyTorch-CPU restatement of the reference's CPU attention -- TEST AND
BASELINE INFRASTRUCTURE ONLY (never the product; only tests/ and bench.py's
CPU-baseline / reference arm use it).

The reference measures its CPU baseline with PyTorch on the host cores
(test.py:39-93 `attention_ref`, timed by test.py:236-252). This module
restates that computation with the same torch operations, in this order:
fp32 upcast, GQA by repeating each KV head over its query-head group
(test.py:66-70), scores = Q K^T * scale (test.py:77), top-left causal mask
via masked_fill of the strict upper triangle with -inf (test.py:80-82),
softmax over the keys, P @ V, (B, S, H, D) layout in and out. Rotate-half
RoPE (common.metal:150-167) is applied to Q and K in fp32 first when asked.
tests/test_oracle.py checks it against the golden fixtures made from the
reference's own function.
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def rope_tables(rows: int, head_dim: int, theta: float):
    """cos/sin [rows, head_dim // 2] float32 from angles computed in float64."""
    i = torch.arange(head_dim // 2, dtype=torch.float64)
    inv_freq = torch.pow(torch.tensor(theta, dtype=torch.float64), -2.0 * i / head_dim)
    ang = torch.arange(rows, dtype=torch.float64)[:, None] * inv_freq[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def rotate_half(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE of x (B, S, H, D) at positions 0..S-1, fp32."""
    x = x.float()
    S, D = x.shape[1], x.shape[3]
    h = D // 2
    c, s = cos[:S, :h][None, :, None, :], sin[:S, :h][None, :, None, :]
    a, b = x[..., :h], x[..., h:2 * h]
    out = x.clone()
    out[..., :h] = a * c - b * s
    out[..., h:2 * h] = a * s + b * c
    return out


@torch.no_grad()
def attention_ref_torch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                        softmax_scale: Optional[float] = None, rope_theta: Optional[float] = None) -> torch.Tensor:
    """O (B, Sq, Hq, D) float32 for CPU tensors q (B, Sq, Hq, D), k/v (B, Sk, Hk, D)."""
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    qf, kf, vf = q.float(), k.float(), v.float()
    if rope_theta:
        cs, sn = rope_tables(max(q.shape[1], k.shape[1]), q.shape[3], rope_theta)
        qf, kf = rotate_half(qf, cs, sn), rotate_half(kf, cs, sn)
    group = q.shape[2] // k.shape[2]
    if group > 1:
        kf = kf.repeat_interleave(group, dim=2)
        vf = vf.repeat_interleave(group, dim=2)
    qh, kh, vh = qf.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2)  # (B, H, S, D)
    scores = torch.matmul(qh, kh.transpose(-2, -1)) * softmax_scale
    if causal:
        Sq, Sk = scores.shape[-2], scores.shape[-1]
        upper = torch.triu(torch.ones(Sq, Sk, dtype=torch.bool), diagonal=1)
        scores = scores.masked_fill(upper, float("-inf"))
    p = torch.softmax(scores, dim=-1)
    return torch.matmul(p, vh).transpose(1, 2).contiguous()
