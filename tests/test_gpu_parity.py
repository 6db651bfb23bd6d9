"""Parity of the CUDA path against the oracle and the reference's golden outputs.

Every test here runs the `_flash_attn_metal` CUDA extension on a B200 and
checks it against (a) fixtures produced by the reference's own attention
oracles (tests/golden) or (b) the NumPy oracle (oracle/attention_oracle.py)
on the same seeded inputs. Bars: fp16/bf16 inputs, float32 output:
max-abs <= 2e-3 and mean-abs <= 2e-4; fp32 inputs: max-abs <= 1e-5 * max|ref|.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import (
    assert_close_16,
    assert_close_32,
    err_stats,
    golden_names,
    load_golden,
)
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _np_dtype(name):
    if name == "bfloat16":
        import ml_dtypes

        return ml_dtypes.bfloat16
    return {"float16": np.float16, "float32": np.float32}[name]


def _torch_dtype(name):
    import torch

    return {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[name]


def _check(got, ref, dtype, what):
    if dtype == "float32":
        return assert_close_32(got, ref, what)
    return assert_close_16(got, ref, what)


@pytest.mark.parametrize("name", golden_names())
def test_golden_numpy_host_path(fa, name):
    g = load_golden(name)
    m = g["meta"]
    dt = _np_dtype(m["dtype"])
    q, k, v = (g[x].astype(dt) for x in ("q", "k", "v"))
    kw = {}
    if "rope_theta" in m:
        kw["rope_theta"] = m["rope_theta"]
    out = fa.forward(q, k, v, softmax_scale=m["scale"], is_causal=m["causal"], out_dtype="float32", **kw)
    assert out.dtype == np.float32 and out.shape == g["out"].shape
    _check(out, g["out"], m["dtype"], name)
    # Default output dtype is the input dtype (float16 in the reference API).
    out_native = fa.forward(q, k, v, softmax_scale=m["scale"], is_causal=m["causal"], **kw)
    assert out_native.dtype == q.dtype
    ulp = {"float16": 2.0**-11, "bfloat16": 2.0**-8, "float32": 2.0**-24}[m["dtype"]]
    d = np.abs(out_native.astype(np.float64) - g["out"])
    assert (d <= 2e-3 + ulp * np.abs(g["out"]) + 1e-7).all(), f"{name}: native-dtype output max_abs={d.max():.3e}"


@pytest.mark.parametrize("name", golden_names())
def test_golden_torch_device_path(fa, cuda_device, name):
    import torch

    g = load_golden(name)
    m = g["meta"]
    tdt = _torch_dtype(m["dtype"])
    q, k, v = (torch.from_numpy(g[x]).to(cuda_device).to(tdt) for x in ("q", "k", "v"))
    kw = {"rope_theta": m["rope_theta"]} if "rope_theta" in m else {}
    n0 = fa.launch_count()
    out, lse = fa.forward(q, k, v, softmax_scale=m["scale"], is_causal=m["causal"], out_dtype="float32",
                          return_lse=True, **kw)
    torch.cuda.synchronize()
    fa.check_status()
    assert fa.launch_count() > n0, "no kernel of the library was launched"
    assert out.is_cuda and out.dtype == torch.float32
    _check(out.cpu().numpy(), g["out"], m["dtype"], name)
    # LSE against the oracle on the same inputs (fp32 math).
    qo, ko = g["q"], g["k"]
    if "rope_theta" in m:
        cs, sn = orc.rope_tables(max(qo.shape[1], ko.shape[1]), qo.shape[3], m["rope_theta"])
        qo, ko = orc.rotate_half_rope(qo, cs, sn), orc.rotate_half_rope(ko, cs, sn)
    _, lse_ref = orc.attention_ref(qo, ko, g["v"], causal=m["causal"], softmax_scale=m["scale"], return_lse=True)
    mx, _ = err_stats(lse.cpu().numpy(), lse_ref)
    assert mx <= 1e-3, f"{name}: LSE max_abs={mx:.3e}"


@pytest.mark.parametrize("name", ["v1_causal_s256_h8_d64", "v2_full_s128_h8_d64"])
def test_verify_correctness_criterion(fa, name):
    """verify_correctness.py:128 bar (max diff < 0.01, no NaN/Inf) against the
    reference's own fp16-cast output, with the reference's call signature."""
    g = load_golden(name)
    q = g["q"].astype(np.float16)
    out = fa.forward(q, q.copy(), q.copy(), softmax_scale=g["meta"]["scale"], is_causal=g["meta"]["causal"])
    assert out.dtype == np.float16
    d = np.abs(out.astype(np.float32) - g["out_f16"].astype(np.float32))
    assert d.max() < 0.01 and np.isfinite(out).all()
    assert_close_16(fa.forward(q, q, q, softmax_scale=g["meta"]["scale"], is_causal=g["meta"]["causal"],
                               out_dtype="float32"), g["out"], name)


# ---------------------------------------------------------------- configs
def _inputs(shape_q, shape_kv, dtype, seed, amp=1.0, device="cuda"):
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    q = (torch.randn(shape_q, generator=gen, device=device) * amp).to(dtype)
    k = (torch.randn(shape_kv, generator=gen, device=device) * amp).to(dtype)
    v = (torch.randn(shape_kv, generator=gen, device=device) * amp).to(dtype)
    return q, k, v


def _oracle_slices(q, k, v, out, lse, causal, scale, theta, heads, row_blocks, group):
    """Compare GPU rows against the oracle for the listed (b, h) pairs and row ranges."""
    import torch

    worst = (0.0, 0.0)
    for b, h in heads:
        hk = h // group
        qh = q[b:b + 1, :, h:h + 1].float().cpu().numpy()
        kh = k[b:b + 1, :, hk:hk + 1].float().cpu().numpy()
        vh = v[b:b + 1, :, hk:hk + 1].float().cpu().numpy()
        if theta:
            cs, sn = orc.rope_tables(max(qh.shape[1], kh.shape[1]), qh.shape[3], theta)
            qh, kh = orc.rotate_half_rope(qh, cs, sn), orc.rotate_half_rope(kh, cs, sn)
        for r0, r1 in row_blocks:
            ref, lse_ref = orc.attention_ref(qh, kh, vh, causal=causal, softmax_scale=scale,
                                             q_range=(r0, r1), return_lse=True)
            got = out[b, r0:r1, h].float().cpu().numpy()
            mx, mean = err_stats(got, ref[0, r0:r1, 0])
            worst = (max(worst[0], mx), max(worst[1], mean))
            assert_close_16(got, ref[0, r0:r1, 0], f"b{b} h{h} rows {r0}:{r1}")
            lmx, _ = err_stats(lse[b, h, r0:r1].float().cpu().numpy(), lse_ref[0, 0, r0:r1])
            assert lmx <= 1e-3, f"LSE b{b} h{h}: {lmx:.3e}"
    return worst


def test_config_readme_fp32_causal(fa, cuda_device):
    """B1 S512 H8 D64 fp32, causal, scale 0.125 (README example shape)."""
    import torch

    q, k, v = _inputs((1, 512, 8, 64), (1, 512, 8, 64), torch.float32, seed=0, device="cuda")
    out = fa.forward(q, k, v, softmax_scale=0.125, is_causal=True)
    ref = orc.attention_ref(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), causal=True, softmax_scale=0.125,
                            compute_dtype=np.float64)
    assert out.dtype == torch.float32
    assert_close_32(out.cpu().numpy(), ref, "fp32 causal")


def test_config_fp16_noncausal_full(fa, cuda_device):
    """B4 S1024 H16 D64 fp16, non-causal, scale 1/8: full comparison."""
    import torch

    q, k, v = _inputs((4, 1024, 16, 64), (4, 1024, 16, 64), torch.float16, seed=1)
    out = fa.forward(q, k, v, softmax_scale=1 / 8, is_causal=False, out_dtype="float32")
    ref = orc.attention_ref(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                            causal=False, softmax_scale=1 / 8)
    assert_close_16(out.cpu().numpy(), ref, "cfg fp16 non-causal")


def test_config_fp16_causal_rope(fa, cuda_device):
    """B8 S2048 H32 D128 fp16, causal, RoPE theta 1e4 (sampled heads, all rows)."""
    import torch

    q, k, v = _inputs((8, 2048, 32, 128), (8, 2048, 32, 128), torch.float16, seed=2)
    out, lse = fa.forward(q, k, v, softmax_scale=1 / math.sqrt(128), is_causal=True, out_dtype="float32",
                          rope_theta=10000.0, return_lse=True)
    torch.cuda.synchronize()
    _oracle_slices(q, k, v, out, lse, True, 1 / math.sqrt(128), 10000.0, [(0, 0), (3, 17), (7, 31)],
                   [(0, 2048)], group=1)


def test_config_bf16_gqa_causal_rope(fa, cuda_device):
    """B4 S8192 Hq32 Hkv8 D128 bf16, causal, RoPE theta 5e5 (sampled heads/rows)."""
    import torch

    q, k, v = _inputs((4, 8192, 32, 128), (4, 8192, 8, 128), torch.bfloat16, seed=3)
    out, lse = fa.forward(q, k, v, softmax_scale=1 / math.sqrt(128), is_causal=True, out_dtype="float32",
                          rope_theta=500000.0, return_lse=True)
    torch.cuda.synchronize()
    fa.check_status()
    _oracle_slices(q, k, v, out, lse, True, 1 / math.sqrt(128), 500000.0, [(0, 0), (1, 13), (3, 31)],
                   [(0, 384), (4000, 4256), (8064, 8192)], group=4)


def test_config_long_context_gqa(fa, cuda_device):
    """B1 S65536 Hq64 Hkv8 D128 bf16 (0.5 * N(0,1)), causal, RoPE theta 5e5 (sampled)."""
    import torch

    q, k, v = _inputs((1, 65536, 64, 128), (1, 65536, 8, 128), torch.bfloat16, seed=4, amp=0.5)
    out, lse = fa.forward(q, k, v, softmax_scale=1 / math.sqrt(128), is_causal=True, out_dtype="float32",
                          rope_theta=500000.0, return_lse=True)
    torch.cuda.synchronize()
    fa.check_status()
    _oracle_slices(q, k, v, out, lse, True, 1 / math.sqrt(128), 500000.0, [(0, 5), (0, 63)],
                   [(0, 128), (30000, 30128), (65408, 65536)], group=8)


# ---------------------------------------------------------------- edge cases
def test_empty_and_degenerate_shapes(fa, cuda_device):
    import torch

    dev = cuda_device
    # No keys: output zeros (softmax over an empty set contributes nothing).
    q = torch.randn(1, 5, 2, 64, device=dev, dtype=torch.float16)
    kv = torch.zeros(1, 0, 2, 64, device=dev, dtype=torch.float16)
    out = fa.forward(q, kv, kv, softmax_scale=0.125)
    assert out.shape == q.shape and torch.count_nonzero(out) == 0
    # Empty batch: empty output.
    e = torch.zeros(0, 16, 2, 64, device=dev, dtype=torch.float16)
    assert fa.forward(e, e, e, softmax_scale=0.1).shape == e.shape
    # One query row, one key.
    q1 = torch.randn(1, 1, 1, 128, device=dev, dtype=torch.bfloat16)
    out1 = fa.forward(q1, q1, q1, softmax_scale=0.1, is_causal=True, out_dtype="float32")
    assert torch.allclose(out1, q1.float(), atol=1e-6)


@pytest.mark.parametrize("S,D,causal", [(1, 64, True), (127, 64, False), (129, 128, True), (1025, 64, True),
                                        (300, 128, False), (97, 96, True), (64, 32, False), (80, 256, True)])
def test_ragged_lengths_and_head_dims(fa, cuda_device, S, D, causal):
    import torch

    q, k, v = _inputs((2, S, 3, D), (2, S, 3, D), torch.float16, seed=S + D)
    out = fa.forward(q, k, v, softmax_scale=1 / math.sqrt(D), is_causal=causal, out_dtype="float32")
    ref = orc.attention_ref(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                            causal=causal, softmax_scale=1 / math.sqrt(D))
    assert_close_16(out.cpu().numpy(), ref, f"S{S} D{D}")


@pytest.mark.parametrize("Sq,Sk", [(64, 300), (300, 64), (200, 513)])
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_cross_attention_top_left_causal(fa, cuda_device, Sq, Sk, dtype):
    import torch

    tdt = _torch_dtype(dtype)
    q, _, _ = _inputs((1, Sq, 4, 128), (1, Sq, 2, 128), tdt, seed=5)
    _, k, v = _inputs((1, Sk, 4, 128), (1, Sk, 2, 128), tdt, seed=6)
    out = fa.forward(q, k, v, softmax_scale=0.09, is_causal=True, out_dtype="float32")
    ref = orc.attention_ref(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                            causal=True, softmax_scale=0.09)
    assert_close_16(out.cpu().numpy(), ref, f"Sq{Sq} Sk{Sk}")


@pytest.mark.parametrize("scale", [0.0, -0.1, 0.3])
def test_unusual_scales(fa, cuda_device, scale):
    """softmax_scale is used as given: 0 gives uniform weights (the reference's
    binding default), negative scales flip the ordering."""
    import torch

    q, k, v = _inputs((1, 200, 2, 64), (1, 200, 2, 64), torch.float16, seed=9)
    out = fa.forward(q, k, v, softmax_scale=scale, is_causal=True, out_dtype="float32")
    ref = orc.attention_ref(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                            causal=True, softmax_scale=scale)
    assert_close_16(out.cpu().numpy(), ref, f"scale {scale}")


def test_strided_head_slice_zero_copy(fa, cuda_device):
    """A head slice of a larger tensor runs in place (strides passed through)."""
    import torch

    q, k, v = _inputs((2, 256, 8, 128), (2, 256, 8, 128), torch.bfloat16, seed=12)
    qs, ks, vs = q[:, :, 2:6], k[:, :, 2:6], v[:, :, 2:6]
    assert not qs.is_contiguous()
    out = fa.forward(qs, ks, vs, softmax_scale=0.1, is_causal=True, out_dtype="float32")
    ref = fa.forward(qs.contiguous(), ks.contiguous(), vs.contiguous(), softmax_scale=0.1, is_causal=True,
                     out_dtype="float32")
    assert torch.equal(out, ref)


def test_cos_sin_tables_match_theta(fa, cuda_device):
    """Explicit cos/sin tables (reference API) give the same result as rope_theta."""
    import torch

    q, k, v = _inputs((1, 384, 4, 128), (1, 384, 4, 128), torch.float16, seed=13)
    cs, sn = orc.rope_tables(384, 128, 10000.0)
    a = fa.forward(q, k, v, softmax_scale=0.088, is_causal=True, cos=cs, sin=sn, out_dtype="float32")
    b = fa.forward(q, k, v, softmax_scale=0.088, is_causal=True, rope_theta=10000.0, out_dtype="float32")
    torch.testing.assert_close(a, b, atol=2e-6, rtol=0)


def test_unaligned_tables_through_c_abi(cuda_device):
    """fa_forward (C ABI) with cos/sin tables 4 bytes off a 16-byte boundary:
    the staging pass reads them element by element (its vector loads need
    16-byte aligned table rows) and gives the aligned tables' result bit for
    bit."""
    import ctypes

    import torch
    from fa_ctypes import FA_BF16, FA_F32, load_lib, make_params

    lib = load_lib()
    B, S, Hq, Hk, D = 1, 640, 4, 2, 128
    q, k, v = _inputs((B, S, Hq, D), (B, S, Hk, D), torch.bfloat16, seed=31)
    cs, sn = orc.rope_tables(S, D, 5e5)
    aligned = [torch.from_numpy(t).to(cuda_device) for t in (cs, sn)]
    shifted = []
    for t in (cs, sn):
        base = torch.zeros(t.size + 1, device=cuda_device)
        view = base[1:].view(t.shape)
        view.copy_(torch.from_numpy(t))
        assert view.data_ptr() % 16 == 4
        shifted.append(view)
    p = make_params(lib, B, S, S, Hq, Hk, D, True, FA_BF16, out_dtype=FA_F32)
    p.has_rotary, p.rope_theta = 1, 0.0  # tables only
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    outs = []
    for c, s in (aligned, shifted):
        o = torch.empty((B, S, Hq, D), dtype=torch.float32, device=cuda_device)
        st = lib.fa_forward(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), None,
                            c.data_ptr(), s.data_ptr(), None, 0, stream)
        assert st == 0, lib.fa_last_error()
        outs.append(o)
    torch.cuda.synchronize()
    assert lib.fa_check_device_status() == 0
    assert torch.equal(outs[0], outs[1])


def test_errors_are_runtime_errors(fa, cuda_device):
    import torch

    q = torch.randn(1, 16, 4, 64, device=cuda_device, dtype=torch.float16)
    k = torch.randn(1, 16, 3, 64, device=cuda_device, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="Forward pass error"):
        fa.forward(q, k, k, softmax_scale=0.1)  # 4 query heads, 3 kv heads
    with pytest.raises(RuntimeError, match="dropout"):
        fa.forward(q, q, q, softmax_scale=0.1, dropout_p=0.1)
    with pytest.raises(RuntimeError, match="alibi_slopes must hold one"):
        fa.forward(q, q, q, softmax_scale=0.1, alibi_slopes=torch.ones(3))


def test_repeated_calls_deterministic(fa, cuda_device):
    import torch

    q, k, v = _inputs((2, 1000, 8, 128), (2, 1000, 2, 128), torch.bfloat16, seed=21)
    a = fa.forward(q, k, v, softmax_scale=0.1, is_causal=True, rope_theta=1e4)
    b = fa.forward(q, k, v, softmax_scale=0.1, is_causal=True, rope_theta=1e4)
    assert torch.equal(a, b)


@pytest.mark.parametrize("B,S,Hq,Hk,dtype,theta", [(3, 4096, 8, 2, "bfloat16", 5e5), (1, 8192, 8, 4, "float16", None),
                                                  (1, 6000, 6, 3, "bfloat16", 1e4),
                                                  (1, 16384, 16, 2, "bfloat16", 5e5),
                                                  (2, 9000, 32, 8, "float16", 1e4)])
def test_host_path_chunked_pipeline_matches_device_path(fa, cuda_device, B, S, Hq, Hk, dtype, theta):
    """Large host-pointer calls are split into (batch, query-row block) chunks
    whose copies overlap compute (heaviest block of each batch first); the
    result must equal the device-path result bit for bit."""
    import torch

    tdt = _torch_dtype(dtype)
    q, k, v = _inputs((B, S, Hq, 128), (B, S, Hk, 128), tdt, seed=B * S + Hq)
    kw = {"rope_theta": theta} if theta else {}
    ref, ref_lse = fa.forward(q, k, v, softmax_scale=0.09, is_causal=True, return_lse=True, **kw)
    qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
    out, lse = fa.forward(qh, kh, vh, softmax_scale=0.09, is_causal=True, return_lse=True, **kw)
    assert not out.is_cuda
    torch.testing.assert_close(out, ref.cpu(), rtol=0, atol=0)
    torch.testing.assert_close(lse, ref_lse.cpu(), rtol=0, atol=0)
    # pageable NumPy arrays take the same path
    if dtype == "float16":
        out_np = fa.forward(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), softmax_scale=0.09, is_causal=True, **kw)
        assert np.array_equal(out_np, ref.cpu().numpy())


@pytest.mark.parametrize("D", [32, 40, 59, 80, 96, 111])
@pytest.mark.parametrize("dtype,causal", [("float16", False), ("bfloat16", True)])
def test_odd_head_dims_padded_onto_tensor_cores(fa, cuda_device, D, dtype, causal):
    """Head dims of the reference's test groups (test.py:293-309,351-368) on
    16-bit inputs run zero-padded on the tensor-core kernel (staging, kernel,
    copy-out: several launches) and match the oracle; with RoPE from cos/sin
    tables, an odd D keeps its last column unrotated."""
    import torch

    q, k, v = _inputs((2, 333, 4, D), (2, 333, 2, D), _torch_dtype(dtype), seed=D)
    kw = {}
    if D % 2 == 1 or D == 80:
        cs, sn = orc.rope_tables(333, D, 10000.0)
        kw = {"cos": torch.from_numpy(cs), "sin": torch.from_numpy(sn)}
    n0 = fa.launch_count()
    out, lse = fa.forward(q, k, v, softmax_scale=1 / math.sqrt(D), is_causal=causal, out_dtype="float32",
                          return_lse=True, **kw)
    torch.cuda.synchronize()
    fa.check_status()
    assert fa.launch_count() - n0 >= 4, "expected the padded tensor-core path (staging, range fixup, kernel, copy-out)"
    qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
    if kw:
        ref, ref_l = orc.attention_with_rope(qn, kn, vn, causal, 1 / math.sqrt(D), cos=cs, sin=sn, return_lse=True)
    else:
        ref, ref_l = orc.attention_ref(qn, kn, vn, causal=causal, softmax_scale=1 / math.sqrt(D), return_lse=True)
    assert_close_16(out.cpu().numpy(), ref, f"D{D} {dtype}")
    assert np.abs(lse.cpu().numpy() - ref_l).max() <= 1e-3
    # the host-pointer path gives the same numbers
    out_h = fa.forward(q.cpu(), k.cpu(), v.cpu(), softmax_scale=1 / math.sqrt(D), is_causal=causal,
                       out_dtype="float32", **kw)
    assert np.array_equal(out_h.numpy(), out.cpu().numpy())


def test_metal_attention_wrapper_with_data(fa, cuda_device):
    """The package wrapper (reference __init__.py:48-89): inputs of any kind
    converted to NumPy float16, scale defaulting to 1/sqrt(head_dim), NumPy
    float16 output equal to the oracle within the fp16 output bar."""
    import torch

    import flash_attn_metal_cpp_b200 as pkg

    rng = np.random.default_rng(8)
    q = rng.standard_normal((2, 200, 4, 64)).astype(np.float32)
    k = rng.standard_normal((2, 200, 2, 64)).astype(np.float32)
    v = rng.standard_normal((2, 200, 2, 64)).astype(np.float32)
    out = pkg.metal_attention(q, k, v, causal=True)
    assert isinstance(out, np.ndarray) and out.dtype == np.float16 and out.shape == q.shape
    q16, k16, v16 = (x.astype(np.float16).astype(np.float32) for x in (q, k, v))
    ref = orc.attention_ref(q16, k16, v16, causal=True, softmax_scale=1 / math.sqrt(64))
    d = np.abs(out.astype(np.float64) - ref)
    assert (d <= 2e-3 + 2.0**-11 * np.abs(ref)).all(), f"max_abs={d.max():.3e}"
    # torch tensors (CUDA or CPU) and nested lists give the same array
    assert np.array_equal(pkg.metal_attention(*(torch.from_numpy(x).to(cuda_device) for x in (q, k, v)),
                                              causal=True), out)
    assert np.array_equal(pkg.metal_attention(q.tolist(), k.tolist(), v.tolist(), causal=True), out)
    # an explicit scale is honoured
    out2 = pkg.metal_attention(q, k, v, causal=False, softmax_scale=0.3)
    ref2 = orc.attention_ref(q16, k16, v16, causal=False, softmax_scale=0.3)
    assert np.abs(out2.astype(np.float64) - ref2).max() <= 2e-3 + 2.0**-11 * np.abs(ref2).max()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("shape", [(2, 300, 4, 2, 64), (2, 5000, 8, 2, 128)])
def test_host_path_pageable_and_pinned_buffers(fa, cuda_device, shape):
    """fa_forward_host with every mix of pageable and pinned host buffers
    (inputs staged by the copy workers, outputs staged on the way back), the
    one-piece and the pipelined path: always the device path's result."""
    import ctypes

    import torch

    from fa_ctypes import FA_F16, FA_F32, load_lib, make_params

    B, S, Hq, Hk, D = shape
    q, k, v = _inputs((B, S, Hq, D), (B, S, Hk, D), torch.float16, seed=S)
    ref, ref_lse = fa.forward(q, k, v, softmax_scale=0.1, is_causal=True, out_dtype="float32", return_lse=True)
    ref, ref_lse = ref.cpu().numpy(), ref_lse.cpu().numpy()
    lib = load_lib()
    lib.fa_forward_host.argtypes = [ctypes.c_void_p] * 8
    lib.fa_forward_host.restype = ctypes.c_int
    p = make_params(lib, B, S, S, Hq, Hk, D, True, FA_F16, FA_F32, scale=0.1)
    for pin_in in (False, True):
        for pin_out in (False, True):
            ins = [x.cpu() for x in (q, k, v)]
            if pin_in:
                ins = [x.pin_memory() for x in ins]
            else:
                ins = [torch.from_numpy(x.numpy().copy()) for x in ins]  # ordinary (pageable) memory
            o = torch.full((B, S, Hq, D), float("nan"))
            lse = torch.full((B, Hq, S), float("nan"))
            if pin_out:
                o, lse = o.pin_memory(), lse.pin_memory()
            st = lib.fa_forward_host(ctypes.addressof(p), *(x.data_ptr() for x in ins), o.data_ptr(), lse.data_ptr(),
                                     None, None)
            assert st == 0, lib.fa_last_error()
            assert np.array_equal(o.numpy(), ref), f"pinned in {pin_in} out {pin_out}"
            assert np.array_equal(lse.numpy(), ref_lse)
