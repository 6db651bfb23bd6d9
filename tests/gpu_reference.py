"""Chunked fp32 evaluation of the oracle's attention formula on the GPU --
TEST INFRASTRUCTURE ONLY (a checker, never the product).

It computes exactly what oracle/attention_oracle.py computes (test.py:39-93
attention_ref: fp32 scores, scale before the top-left causal mask, softmax
over keys, P @ V; GQA by kv_head = q_head // group; rotate-half RoPE of
common.metal:150-167 with the oracle's float64-built tables), but with
torch fp32 matmuls on the GPU (TF32 off), per (batch, KV head) and per
block of query rows, so whole outputs of the full-size configurations
(up to S = 65536) can be checked element by element in seconds. The tests
validate it against the NumPy oracle on slices before trusting it.
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch

from oracle import attention_oracle as orc


def rope_fp32(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE of x (B, S, H, D) in fp32 at positions 0..S-1."""
    x = x.float()
    S, D = x.shape[1], x.shape[3]
    h = D // 2
    c = cos[:S, :h][None, :, None, :]
    s = sin[:S, :h][None, :, None, :]
    out = x.clone()
    a, b = x[..., :h], x[..., h:2 * h]
    out[..., :h] = a * c - b * s
    out[..., h:2 * h] = a * s + b * c
    return out


@torch.no_grad()
def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, scale: float,
                   theta: Optional[float] = None, row_block: int = 4096,
                   q_range: Optional[Tuple[int, int]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(O, LSE): O (B, Sq, Hq, D) fp32, LSE (B, Hq, Sq) fp32 (natural log).

    q, k, v are CUDA tensors of any float dtype (their values are taken
    exactly). Rows outside q_range are left at 0 / -inf."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        B, Sq, Hq, D = q.shape
        Sk, Hk = k.shape[1], k.shape[2]
        g = Hq // Hk
        dev = q.device
        if theta:
            c_np, s_np = orc.rope_tables(max(Sq, Sk), D, theta)
            cs, sn = torch.from_numpy(c_np).to(dev), torch.from_numpy(s_np).to(dev)
        out = torch.zeros((B, Sq, Hq, D), dtype=torch.float32, device=dev)
        lse = torch.full((B, Hq, Sq), float("-inf"), dtype=torch.float32, device=dev)
        r_lo, r_hi = (0, Sq) if q_range is None else q_range
        keys = torch.arange(Sk, device=dev)
        for b in range(B):
            kb, vb = k[b:b + 1].float(), v[b].float()
            if theta:
                kb = rope_fp32(kb, cs, sn)
            kb = kb[0]
            for hk in range(Hk):
                kh = kb[:, hk]                       # (Sk, D)
                vh = vb[:, hk]
                qg = q[b:b + 1, :, hk * g:(hk + 1) * g].float()
                if theta:
                    qg = rope_fp32(qg, cs, sn)
                qg = qg[0].permute(1, 0, 2)          # (g, Sq, D)
                for r0 in range(r_lo, r_hi, row_block):
                    r1 = min(r_hi, r0 + row_block)
                    qh = qg[:, r0:r1]                # (g, R, D)
                    kend = min(Sk, r1) if causal else Sk
                    if kend == 0:
                        continue
                    s = torch.matmul(qh, kh[:kend].t()) * scale  # (g, R, kend)
                    if causal:
                        rows = torch.arange(r0, r1, device=dev)
                        s.masked_fill_((keys[None, :kend] > rows[:, None])[None], float("-inf"))
                    m = s.amax(dim=2, keepdim=True)
                    p = torch.exp(s - m)
                    l = p.sum(dim=2, keepdim=True)
                    o = torch.matmul(p, vh[:kend]) / l  # (g, R, D)
                    out[b, r0:r1, hk * g:(hk + 1) * g] = o.permute(1, 0, 2)
                    lse[b, hk * g:(hk + 1) * g, r0:r1] = (m + torch.log(l))[..., 0]
                    del s, p
        return out, lse
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def compare_whole(got: torch.Tensor, ref: torch.Tensor, max_abs: float, mean_abs: float, what: str):
    """Every element: max |got - ref| <= max_abs, mean <= mean_abs, all finite.
    Returns (max, mean) as floats."""
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    d = (got.float() - ref).abs()
    mx, mean = float(d.max()), float(d.mean(dtype=torch.float64))
    assert mx <= max_abs and mean <= mean_abs, f"{what}: max_abs={mx:.3e} mean_abs={mean:.3e}"
    return mx, mean


def oracle_slice(q, k, v, causal, scale, theta, b, h, rows):
    """NumPy-oracle rows of one (batch, query head) for validating attention_fp32."""
    g = q.shape[2] // k.shape[2]
    hk = h // g
    qh = q[b:b + 1, :, h:h + 1].float().cpu().numpy()
    kh = k[b:b + 1, :, hk:hk + 1].float().cpu().numpy()
    vh = v[b:b + 1, :, hk:hk + 1].float().cpu().numpy()
    if theta:
        cs, sn = orc.rope_tables(max(qh.shape[1], kh.shape[1]), qh.shape[3], theta)
        qh, kh = orc.rotate_half_rope(qh, cs, sn), orc.rotate_half_rope(kh, cs, sn)
    o, l = orc.attention_ref(qh, kh, vh, causal=causal, softmax_scale=scale, q_range=rows, return_lse=True)
    return np.asarray(o[0, rows[0]:rows[1], 0]), np.asarray(l[0, 0, rows[0]:rows[1]])
