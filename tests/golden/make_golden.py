"""Generate the golden attention fixtures from the reference's own oracles.

Run in a container where the reference checkout is mounted (read-only is
fine):  python tests/golden/make_golden.py <reference checkout>

It imports `attention_ref` (test.py:39-93) and `torch_attention_reference`
(verify_correctness.py:34-66) from the reference with a stub
`_flash_attn_metal` module in sys.modules (the Metal extension cannot be
built off macOS; the oracles are plain torch CPU code), runs them on seeded
inputs built the way the reference tests build them, and writes one .npz per
case next to this script. Inputs are stored in their own format (float16,
float32, or bfloat16 as uint16 bit patterns); `out` is the reference
oracle's float32 output. The fixtures are small so they can be committed.

RoPE cases: the reference never applies RoPE in a test, so the rotation here
is a torch transcription of common.metal:150-167 (pairs (i, i + D/2)), applied
to Q and K before calling the reference's attention_ref.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _stub_module():
    stub = types.ModuleType("_flash_attn_metal")
    stub.initialize = lambda: True
    stub.compile_shaders = lambda src: True
    stub.load_shaders = lambda path: True
    stub.get_device_info = lambda: {}

    def _no_forward(*a, **k):
        raise RuntimeError("stub: the Metal kernel is not available here")

    stub.forward = _no_forward
    return stub


def load_reference(ref_dir: str):
    sys.modules["_flash_attn_metal"] = _stub_module()
    cwd = os.getcwd()
    os.chdir(ref_dir)  # verify_correctness.py reads kernels/*.metal relative to the cwd
    try:
        mods = {}
        for name, fname in (("ref_test", "test.py"), ("ref_verify", "verify_correctness.py")):
            spec = importlib.util.spec_from_file_location(name, os.path.join(ref_dir, fname))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mods[name] = mod
    finally:
        os.chdir(cwd)
    return mods["ref_test"].attention_ref, mods["ref_verify"].torch_attention_reference


def rope_torch(x: torch.Tensor, theta: float) -> torch.Tensor:
    """Transcription of common.metal:150-167 with tables angle = pos * theta^(-2i/D)."""
    B, S, H, D = x.shape
    half = D // 2
    i = torch.arange(half, dtype=torch.float64)
    inv = torch.pow(torch.tensor(theta, dtype=torch.float64), -2.0 * i / D)
    ang = torch.arange(S, dtype=torch.float64)[:, None] * inv[None, :]
    c = torch.cos(ang).float()[None, :, None, :]
    s = torch.sin(ang).float()[None, :, None, :]
    xf = x.float()
    a, b = xf[..., :half], xf[..., half:2 * half]
    out = xf.clone()
    out[..., :half] = a * c - b * s
    out[..., half:2 * half] = a * s + b * c
    return out


def _native(t: torch.Tensor) -> np.ndarray:
    """Inputs in their own 16/32-bit format; bfloat16 as its uint16 bit pattern."""
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def save(name, q, k, v, out, meta, extra=None):
    if k is q and v is q:  # k = v = q (verify_correctness.py:75-76): store q once
        arrays = dict(q=_native(q), out=out)
        meta = dict(meta, kv_is_q=True)
    else:
        arrays = dict(q=_native(q), k=_native(k), v=_native(v), out=out)
    if extra:
        arrays.update(extra)
    meta = dict(meta, name=name)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), meta=json.dumps(meta), **arrays)
    print(name, {k2: v2.shape for k2, v2 in arrays.items()})


def main(ref_dir: str) -> None:
    attention_ref, torch_attention_reference = load_reference(ref_dir)
    gen = "reference test.py attention_ref"

    # Cases shaped like test.py test_correctness (:126-180): torch seed 42,
    # randn * 0.02 in float16, separate q/k/v, scale 1/sqrt(D), non-causal.
    testpy_cases = [
        ("t1_basic_b2_s97_h3_d64", 2, 97, 97, 3, 3, 64),
        ("t2_nonsquare_q113_k203_d32", 1, 113, 203, 3, 3, 32),
        ("t3_gqa_h8kv2_s128_d64", 1, 128, 128, 8, 2, 64),
        ("t4_mqa_h8kv1_s64_d128", 1, 64, 64, 8, 1, 128),
        ("t5_edge_s97_d59", 1, 97, 97, 2, 2, 59),
        ("t6_edge_s200_d40", 1, 200, 200, 2, 2, 40),
        ("t7_nonsquare_q128_k320_d128", 1, 128, 320, 1, 1, 128),
    ]
    for name, B, Sq, Sk, Hq, Hk, D in testpy_cases:
        torch.manual_seed(42)
        q = torch.randn(B, Sq, Hq, D, dtype=torch.float16) * 0.02
        k = torch.randn(B, Sk, Hk, D, dtype=torch.float16) * 0.02
        v = torch.randn(B, Sk, Hk, D, dtype=torch.float16) * 0.02
        scale = 1.0 / np.sqrt(D)
        out = attention_ref(q, k, v, causal=False, softmax_scale=scale).numpy().astype(np.float32)
        save(name, q, k, v, out, dict(dtype="float16", causal=False, scale=float(scale), generator=gen))

    # Shaped like verify_correctness.py (:69-94): numpy seed 42, q = randn * 0.02
    # in float16, k = v = q; output of the reference's fp16-casting oracle.
    for name, S, causal in (("v1_causal_s256_h8_d64", 256, True), ("v2_full_s128_h8_d64", 128, False)):
        np.random.seed(42)
        qn = np.random.randn(1, S, 8, 64).astype(np.float16) * 0.02
        scale = 1.0 / np.sqrt(64)
        out16 = torch_attention_reference(qn, qn.copy(), qn.copy(), scale, causal)
        qt = torch.from_numpy(qn)
        out32 = attention_ref(qt, qt, qt, causal=causal, softmax_scale=scale).numpy().astype(np.float32)
        save(name, qt, qt, qt, out32,
             dict(dtype="float16", causal=causal, scale=float(scale),
                  generator="reference verify_correctness.py torch_attention_reference + test.py attention_ref"),
             extra=dict(out_f16=out16))

    # Causal, top-left aligned, Sq != Sk (test.py:80-82 mask), and the fp32
    # configuration of the README example (scale 0.125) at a small size.
    torch.manual_seed(7)
    for name, Sq, Sk in (("c1_causal_q64_k100_d64", 64, 100), ("c2_causal_q100_k64_d64", 100, 64)):
        q = torch.randn(1, Sq, 2, 64, dtype=torch.float16)
        k = torch.randn(1, Sk, 2, 64, dtype=torch.float16)
        v = torch.randn(1, Sk, 2, 64, dtype=torch.float16)
        out = attention_ref(q, k, v, causal=True, softmax_scale=0.125).numpy().astype(np.float32)
        save(name, q, k, v, out, dict(dtype="float16", causal=True, scale=0.125, generator=gen))
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 128, 2, 64, generator=g)
    k = torch.randn(1, 128, 2, 64, generator=g)
    v = torch.randn(1, 128, 2, 64, generator=g)
    out = attention_ref(q, k, v, causal=True, softmax_scale=0.125).numpy().astype(np.float32)
    save("f1_fp32_causal_s128_h2_d64", q, k, v, out, dict(dtype="float32", causal=True, scale=0.125, generator=gen))

    # bf16 GQA causal, N(0,1) inputs (the long-context configuration's format).
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 192, 4, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 192, 1, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, 192, 1, 128, generator=g).to(torch.bfloat16)
    out = attention_ref(q.float(), k.float(), v.float(), causal=True,
                        softmax_scale=1 / np.sqrt(128)).numpy().astype(np.float32)
    save("b1_bf16_gqa_causal_s192_h4kv1_d128", q, k, v, out,
         dict(dtype="bfloat16", causal=True, scale=float(1 / np.sqrt(128)), generator=gen))

    # RoPE (rotate-half, common.metal:150-167) then the reference attention_ref.
    for name, dtype, theta, Hq, Hk, S, D in (
        ("r1_rope_f16_causal_s128_h2_d128_t1e4", torch.float16, 10000.0, 2, 2, 128, 128),
        ("r2_rope_bf16_gqa_causal_s160_h4kv2_d128_t5e5", torch.bfloat16, 500000.0, 4, 2, 160, 128),
        ("r3_rope_f16_causal_s96_h2_d64_t1e4", torch.float16, 10000.0, 2, 2, 96, 64),
    ):
        g = torch.Generator().manual_seed(11)
        q = torch.randn(1, S, Hq, D, generator=g).to(dtype)
        k = torch.randn(1, S, Hk, D, generator=g).to(dtype)
        v = torch.randn(1, S, Hk, D, generator=g).to(dtype)
        scale = 1.0 / np.sqrt(D)
        out = attention_ref(rope_torch(q, theta), rope_torch(k, theta), v.float(), causal=True,
                            softmax_scale=scale).numpy().astype(np.float32)
        save(name, q, k, v, out,
             dict(dtype=str(dtype).replace("torch.", ""), causal=True, scale=float(scale), rope_theta=theta,
                  generator="torch transcription of common.metal:150-167 + reference test.py attention_ref"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
