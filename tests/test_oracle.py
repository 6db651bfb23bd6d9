"""The oracle against the reference's golden vectors, plus its own properties (CPU)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_names, load_golden
from oracle import attention_oracle as orc


def _oracle_out(g):
    m = g["meta"]
    if "rope_theta" in m:
        return orc.attention_with_rope(g["q"], g["k"], g["v"], causal=m["causal"], softmax_scale=m["scale"],
                                       theta=m["rope_theta"])
    return orc.attention_ref(g["q"], g["k"], g["v"], causal=m["causal"], softmax_scale=m["scale"])


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_fixture(name):
    g = load_golden(name)
    got = _oracle_out(g)
    ref = g["out"]
    scale = float(np.abs(ref).max())
    assert np.abs(got - ref).max() <= 1e-5 * scale + 1e-7, name


@pytest.mark.parametrize("name", golden_names())
def test_torch_cpu_baseline_matches_reference_fixture(name):
    """The PyTorch-CPU restatement timed as the CPU baseline computes what the
    reference's attention_ref computed for the fixtures."""
    import torch

    from oracle.torch_cpu_reference import attention_ref_torch

    g = load_golden(name)
    m = g["meta"]
    q, k, v = (torch.from_numpy(g[x]) for x in ("q", "k", "v"))
    got = attention_ref_torch(q, k, v, causal=m["causal"], softmax_scale=m["scale"],
                              rope_theta=m.get("rope_theta")).numpy()
    scale = float(np.abs(g["out"]).max())
    assert np.abs(got - g["out"]).max() <= 1e-5 * scale + 1e-7, name


@pytest.mark.parametrize("name", ["v1_causal_s256_h8_d64", "v2_full_s128_h8_d64"])
def test_fp16_cast_oracle_matches_verify_correctness(name):
    """torch_attention_reference (verify_correctness.py:34-66) returns fp16."""
    g = load_golden(name)
    q = g["q"].astype(np.float16)
    got = orc.torch_attention_reference(q, q, q, g["meta"]["scale"], g["meta"]["causal"])
    assert got.dtype == np.float16
    d = np.abs(got.astype(np.float32) - g["out_f16"].astype(np.float32))
    ulp = np.spacing(np.abs(g["out_f16"]).astype(np.float16)).astype(np.float32)
    assert (d <= ulp).all()


def test_planted_bottom_right_mask_is_caught():
    """A wrong causal alignment in the oracle (bottom-right, as upstream FA2)
    must disagree with the reference fixtures for Sq != Sk."""
    g = load_golden("c1_causal_q64_k100_d64")
    q, k, v = g["q"], g["k"], g["v"]
    Sq, Sk = q.shape[1], k.shape[1]
    # bottom-right alignment == top-left with queries shifted by Sk - Sq
    qs = np.zeros((1, Sk, 2, 64), np.float32)
    qs[:, Sk - Sq:] = q
    wrong = orc.attention_ref(qs, k, v, causal=True, softmax_scale=0.125)[:, Sk - Sq:]
    assert np.abs(wrong - g["out"]).max() > 1e-2
    assert np.abs(_oracle_out(g) - g["out"]).max() < 1e-5


def test_gqa_equals_repeated_heads():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 40, 6, 32), dtype=np.float32)
    k = rng.standard_normal((2, 50, 2, 32), dtype=np.float32)
    v = rng.standard_normal((2, 50, 2, 32), dtype=np.float32)
    a = orc.attention_ref(q, k, v, causal=True, softmax_scale=0.2)
    b = orc.attention_ref(q, np.repeat(k, 3, axis=2), np.repeat(v, 3, axis=2), causal=True, softmax_scale=0.2)
    np.testing.assert_allclose(a, b, rtol=0, atol=1e-6)


def test_split_partials_combine_to_full():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 300, 2, 16), dtype=np.float32)
    k = rng.standard_normal((1, 300, 1, 16), dtype=np.float32)
    v = rng.standard_normal((1, 300, 1, 16), dtype=np.float32)
    full, lse = orc.attention_ref(q, k, v, causal=True, softmax_scale=0.3, return_lse=True)
    parts = [orc.attention_ref(q, k, v, causal=True, softmax_scale=0.3, return_lse=True, kv_range=r)
             for r in [(0, 37), (37, 150), (150, 300)]]
    o, l = orc.combine_partials([p[0] for p in parts], [p[1] for p in parts])
    np.testing.assert_allclose(o, full, atol=2e-6)
    np.testing.assert_allclose(l, lse, atol=2e-5)
    # a range no row can see (rows < 150 see no key >= 150) gives O = 0, LSE = -inf there
    p3 = parts[2]
    assert np.all(p3[1][0, :, :150] == -np.inf) and np.all(p3[0][0, :150] == 0)


def test_rope_tables_and_rotation():
    cs, sn = orc.rope_tables(10, 8, 10000.0)
    assert cs.shape == (10, 4) and cs.dtype == np.float32
    np.testing.assert_allclose(cs[0], 1.0)
    np.testing.assert_allclose(sn[0], 0.0)
    np.testing.assert_allclose(np.arctan2(sn[3, 1], cs[3, 1]), 3 * 10000.0 ** (-2 / 8), rtol=1e-6)
    x = np.random.default_rng(2).standard_normal((1, 10, 1, 9), dtype=np.float32)  # odd D: last col kept
    y = orc.rotate_half_rope(x, *orc.rope_tables(10, 9, 100.0))
    np.testing.assert_array_equal(y[..., 8], x[..., 8])
    np.testing.assert_allclose(np.linalg.norm(y[..., :8], axis=-1), np.linalg.norm(x[..., :8], axis=-1), rtol=1e-5)


def test_empty_keys_and_uniform_scale():
    q = np.ones((1, 3, 1, 4), np.float32)
    e = np.zeros((1, 0, 1, 4), np.float32)
    assert np.all(orc.attention_ref(q, e, e, softmax_scale=1.0) == 0)
    rng = np.random.default_rng(3)
    k = rng.standard_normal((1, 5, 1, 4), dtype=np.float32)
    v = rng.standard_normal((1, 5, 1, 4), dtype=np.float32)
    out = orc.attention_ref(np.ones((1, 5, 1, 4), np.float32), k, v, causal=True, softmax_scale=0.0)
    np.testing.assert_allclose(out[0, 4, 0], v[0, :, 0].mean(axis=0), atol=1e-6)  # uniform weights
    np.testing.assert_allclose(out[0, 0, 0], v[0, 0, 0], atol=1e-6)


def test_flop_count_convention():
    assert orc.attention_flops(4, 8192, 8192, 32, 128, True) == 4 * 4 * 32 * 8192 * 8192 * 128 / 2


@pytest.mark.parametrize("causal,window,alibi", [(True, (7, -1), True), (False, (5, 3), False),
                                                 (False, None, True), (True, (-1, -1), False)])
def test_window_and_alibi_match_dense_formula(causal, window, alibi):
    """Sliding window (common.metal:95-104) and ALiBi (common.metal:123-128)
    against a dense torch evaluation of the same formulas."""
    import torch

    rng = np.random.default_rng(11)
    B, Sq, Sk, H, D = 2, 37, 45, 3, 16
    q = rng.standard_normal((B, Sq, H, D), dtype=np.float32)
    k = rng.standard_normal((B, Sk, H, D), dtype=np.float32)
    v = rng.standard_normal((B, Sk, H, D), dtype=np.float32)
    sl = np.array([0.5, 0.25, 0.125], np.float32) if alibi else None
    got = orc.attention_ref(q, k, v, causal=causal, softmax_scale=0.3, window=window, alibi_slopes=sl, q_block=8)
    qt, kt, vt = (torch.from_numpy(x).permute(0, 2, 1, 3).double() for x in (q, k, v))
    s = qt @ kt.transpose(-1, -2) * 0.3
    rel = (torch.arange(Sk)[None, :] - torch.arange(Sq)[:, None]).double()
    if alibi:
        s = s + torch.from_numpy(sl).double()[None, :, None, None] * rel
    mask = torch.zeros(Sq, Sk, dtype=torch.bool)
    if causal:
        mask |= rel > 0
    if window is not None and window[0] >= 0:
        mask |= rel < -window[0]
    if window is not None and window[1] >= 0:
        mask |= rel > window[1]
    s = s.masked_fill(mask, -float("inf"))
    p = torch.softmax(s, -1).nan_to_num(0.0)
    ref = (p @ vt).permute(0, 2, 1, 3).numpy()
    np.testing.assert_allclose(got, ref, atol=2e-6)
