"""CPU oracle for the attention forward path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only tests/, the smoke()
entry point and bench.py's CPU-baseline / reference arm may import it. The
product path (the `_flash_attn_metal` extension) never calls it and has no
CPU fallback.

It restates, in NumPy, the reference's CPU attention oracles:
  * attention_ref            test.py:39-93 (fp32 math, GQA by repeating KV heads
                             test.py:66-70, scale before mask test.py:77,
                             top-left causal mask triu(diagonal=1) test.py:80-82,
                             softmax over keys, P @ V, (B, S, H, D) layout)
  * torch_attention_reference verify_correctness.py:34-66 (same math, square
                             causal mask :54, output cast to float16 :66)
plus the parts of the path the reference only declares:
  * rotate_half_rope         common.metal:150-167 (pairs (i, i + D/2);
                             x' = x cos - y sin, y' = x sin + y cos;
                             table index pos * (D/2) + i)
  * rope_tables              [rows, D/2] float32 cos/sin tables, the layout the
                             reference host binds (src/flash_attn_core.cpp:343-349),
                             angle(pos, i) = pos * theta^(-2i/D) computed in float64
  * gqa head map             common.metal:215-217 (kv_head = q_head // group)
  * sliding-window mask      common.metal:95-104 (key k masked for query q iff
                             window_left >= 0 and k - q < -window_left, or
                             window_right >= 0 and k - q > window_right;
                             combined with the causal mask, :107-119)
  * ALiBi bias               common.metal:123-128 (slope[h] * (k - q) added to
                             the scaled score)
and the split-KV partial / (O, LSE) combine used by the multi-GPU path.

Pinning: attention_ref / torch_attention_reference are checked against
fixtures produced by the reference's own functions (tests/golden/, made by
tests/golden/make_golden.py, which imports test.py and verify_correctness.py
from the reference). RoPE has no reference test; its fixtures come from a
torch transcription of common.metal:150-167 fed into the reference's
attention_ref, so the rotation formula is pinned only by that transcription.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np


def rope_tables(rows: int, head_dim: int, theta: float) -> Tuple[np.ndarray, np.ndarray]:
    """cos/sin tables [rows, head_dim // 2] float32; angle = pos * theta**(-2i/head_dim)."""
    half = head_dim // 2
    i = np.arange(half, dtype=np.float64)
    inv_freq = np.power(np.float64(theta), -2.0 * i / np.float64(head_dim))
    ang = np.arange(rows, dtype=np.float64)[:, None] * inv_freq[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rotate_half_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE of x (B, S, H, D) at positions 0..S-1 (common.metal:150-167).

    Returns float32. For odd D the last column has no partner and is kept.
    """
    x = np.asarray(x, dtype=np.float32)
    S, D = x.shape[1], x.shape[3]
    h = D // 2
    c = cos[:S, :h][None, :, None, :].astype(np.float32)
    s = sin[:S, :h][None, :, None, :].astype(np.float32)
    out = x.copy()
    a = x[..., :h]
    b = x[..., h : 2 * h]
    out[..., :h] = a * c - b * s
    out[..., h : 2 * h] = a * s + b * c
    return out


def _scores_block(q_blk: np.ndarray, k_bh: np.ndarray, scale: float) -> np.ndarray:
    return (q_blk @ k_bh.T) * np.float32(scale)


def attention_ref(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    causal: bool = False,
    softmax_scale: Optional[float] = None,
    *,
    return_lse: bool = False,
    q_block: int = 1024,
    compute_dtype=np.float32,
    kv_range: Optional[Tuple[int, int]] = None,
    q_range: Optional[Tuple[int, int]] = None,
    window: Optional[Tuple[int, int]] = None,
    alibi_slopes: Optional[np.ndarray] = None,
):
    """NumPy restatement of test.py:39-93 `attention_ref`.

    window=(left, right) adds the sliding-window mask of common.metal:95-104
    (a negative side is unbounded); alibi_slopes (Hq,) adds
    slope[h] * (k - q) to the scaled scores (common.metal:123-128).

    q: (B, Sq, Hq, D), k/v: (B, Sk, Hk, D), any float dtype (values are
    taken exactly, then computed in `compute_dtype`, float32 by default as
    in the reference). Returns O (B, Sq, Hq, D) in compute_dtype and, with
    return_lse, LSE (B, Hq, Sq) (natural log).

    Evaluated per (batch, head) and per block of `q_block` query rows so
    large sequence lengths never materialise a full score matrix.

    kv_range=(lo, hi) restricts the keys to [lo, hi) (split-KV partial; rows
    with no visible key give O = 0, LSE = -inf); q_range=(lo, hi) computes
    only those rows (others are left as zero / -inf).
    """
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    B, Sq, Hq, D = q.shape
    _, Sk, Hk, _ = k.shape
    assert Hq % Hk == 0, "num_heads_q must be a multiple of num_heads_k"
    group = Hq // Hk
    cd = compute_dtype
    qf = np.asarray(q).astype(cd)
    kf = np.asarray(k).astype(cd)
    vf = np.asarray(v).astype(cd)
    out = np.zeros((B, Sq, Hq, D), dtype=cd)
    lse = np.full((B, Hq, Sq), -np.inf, dtype=cd)
    k_lo, k_hi = (0, Sk) if kv_range is None else kv_range
    r_lo, r_hi = (0, Sq) if q_range is None else q_range
    if k_hi <= k_lo:  # no key at all: softmax over an empty set contributes nothing
        return (out, lse) if return_lse else out
    keys = np.arange(Sk)
    for b in range(B):
        for h in range(Hq):
            hk = h // group  # common.metal:215-217 / repeat_interleave in test.py:69
            k_bh = kf[b, :, hk, :]
            v_bh = vf[b, :, hk, :]
            for r0 in range(r_lo, r_hi, q_block):
                r1 = min(r0 + q_block, r_hi)
                s = _scores_block(qf[b, r0:r1, h, :], k_bh, softmax_scale)
                vis = (keys[None, :] >= k_lo) & (keys[None, :] < k_hi)
                rel = keys[None, :] - np.arange(r0, r1)[:, None]  # k - q
                if causal:  # top-left: key k masked for query q iff k > q (triu diagonal=1)
                    vis = vis & (rel <= 0)
                if window is not None:  # common.metal:95-104
                    wl, wr = window
                    if wl >= 0:
                        vis = vis & (rel >= -wl)
                    if wr >= 0:
                        vis = vis & (rel <= wr)
                if alibi_slopes is not None:  # common.metal:123-128
                    s = s + (np.float32(alibi_slopes[h]) * rel.astype(np.float32)).astype(cd)
                vis = np.broadcast_to(vis, s.shape)
                s = np.where(vis, s, -np.inf)
                m = s.max(axis=1, keepdims=True)
                any_vis = np.isfinite(m)
                m_safe = np.where(any_vis, m, 0).astype(cd)
                p = np.where(vis, np.exp(s - m_safe), 0).astype(cd)
                l = p.sum(axis=1, keepdims=True)
                with np.errstate(divide="ignore", invalid="ignore"):
                    o = np.where(any_vis, (p @ v_bh) / np.where(l > 0, l, 1), 0)
                    lse_blk = np.where(any_vis[:, 0], m_safe[:, 0] + np.log(np.where(l[:, 0] > 0, l[:, 0], 1)), -np.inf)
                out[b, r0:r1, h, :] = o
                lse[b, h, r0:r1] = lse_blk
    if return_lse:
        return out, lse
    return out


def torch_attention_reference(q: np.ndarray, k: np.ndarray, v: np.ndarray, softmax_scale: float,
                              is_causal: bool = False) -> np.ndarray:
    """NumPy restatement of verify_correctness.py:34-66 (fp32 math, fp16 output)."""
    return attention_ref(q, k, v, causal=is_causal, softmax_scale=softmax_scale).astype(np.float16)


def attention_with_rope(q, k, v, causal, softmax_scale, theta=None, cos=None, sin=None, **kw):
    """Rotate Q and K (fp32) with rotate-half RoPE, then attention_ref."""
    if cos is None:
        cos, sin = rope_tables(max(q.shape[1], k.shape[1]), q.shape[3], theta)
    qr = rotate_half_rope(q, cos, sin)
    kr = rotate_half_rope(k, cos, sin)
    return attention_ref(qr, kr, v, causal=causal, softmax_scale=softmax_scale, **kw)


def combine_partials(o_parts, lse_parts):
    """Merge split-KV partials: LSE = log sum exp(LSE_j), O = sum exp(LSE_j - LSE) O_j.

    o_parts: (n, B, S, H, D); lse_parts: (n, B, H, S). Rows where every
    partial is empty (-inf) give O = 0 and LSE = -inf.
    """
    o_parts = np.asarray(o_parts, dtype=np.float64)
    lse_parts = np.asarray(lse_parts, dtype=np.float64)
    mx = lse_parts.max(axis=0)
    finite = np.isfinite(mx)
    mx_safe = np.where(finite, mx, 0)
    w = np.where(np.isfinite(lse_parts), np.exp(lse_parts - mx_safe[None]), 0)
    wsum = w.sum(axis=0)
    with np.errstate(divide="ignore"):
        lse = np.where(wsum > 0, mx_safe + np.log(np.where(wsum > 0, wsum, 1)), -np.inf)
    coef = np.where(wsum[None] > 0, w / np.where(wsum > 0, wsum, 1)[None], 0)  # (n, B, H, S)
    o = np.einsum("nbhs,nbshd->bshd", coef, o_parts)
    return o, lse


def attention_flops(B: int, Sq: int, Sk: int, Hq: int, D: int, causal: bool) -> float:
    """Headline FLOP count 4*B*H*Sq*Sk*D, halved for causal (softmax and RoPE not counted)."""
    f = 4.0 * B * Hq * Sq * Sk * D
    return f / 2 if causal else f
