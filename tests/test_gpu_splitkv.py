"""Split-KV building blocks on the GPU against the oracle.

* forward_range: rows [q0, q1) over keys [k0, k1) -- partial (O, LSE) with
  absolute positions for RoPE and the causal mask; rows outside the query
  range are not written.
* routed epilogue: the same partial written into per-owner staging slots
  through a device address table (single process, local slots).
* combine: the merge of split partials equals attention over all keys.
* SplitKVAttention on two GPUs (one process each, NCCL + CUDA IPC): each
  rank's owned rows against the oracle; skipped with fewer than two GPUs.

Bars as elsewhere: 16-bit inputs with float32 output max-abs <= 2e-3 and
mean-abs <= 2e-4; LSE max-abs <= 1e-3; fp32 inputs 1e-5 relative.
"""
from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest

from conftest import assert_close_16, assert_close_32, err_stats
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(shape_q, shape_kv, dtype, seed, amp=1.0, device="cuda"):
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    q = (torch.randn(shape_q, generator=gen, device=device) * amp).to(dtype)
    k = (torch.randn(shape_kv, generator=gen, device=device) * amp).to(dtype)
    v = (torch.randn(shape_kv, generator=gen, device=device) * amp).to(dtype)
    return q, k, v


def _np(t):
    return t.float().cpu().numpy()


def _oracle(q, k, v, causal, scale, theta, **kw):
    qn, kn, vn = _np(q), _np(k), _np(v)
    if theta:
        return orc.attention_with_rope(qn, kn, vn, causal, scale, theta=theta, return_lse=True, **kw)
    return orc.attention_ref(qn, kn, vn, causal=causal, softmax_scale=scale, return_lse=True, **kw)


def _check_rows(got_o, got_l, ref_o, ref_l, rows, fp32, what):
    r0, r1 = rows
    go, ro = got_o[:, r0:r1], ref_o[:, r0:r1]
    if fp32:
        assert_close_32(go, ro, what)
    else:
        assert_close_16(go, ro, what)
    gl, rl = got_l[:, :, r0:r1], ref_l[:, :, r0:r1]
    assert np.array_equal(np.isneginf(gl), np.isneginf(rl)), f"{what}: LSE -inf pattern differs"
    fin = np.isfinite(rl)
    if fin.any():
        assert np.abs(gl[fin] - rl[fin]).max() <= 1e-3, f"{what}: LSE"


@pytest.mark.parametrize(
    "B,S,Hq,Hk,D,dtype,causal,theta,q_range,kv_range",
    [
        (2, 700, 4, 2, 128, "bfloat16", True, 1e4, (128, 640), (256, 600)),
        (1, 1000, 8, 1, 128, "bfloat16", True, 5e5, (0, 1000), (384, 1000)),
        (2, 513, 4, 4, 64, "float16", False, None, (100, 513), (0, 200)),
        (1, 300, 2, 1, 40, "float32", True, None, (17, 300), (50, 290)),
        (1, 256, 2, 2, 128, "float16", True, None, (0, 128), (128, 256)),  # no visible key
    ],
)
def test_forward_range_matches_oracle(fa, cuda_device, B, S, Hq, Hk, D, dtype, causal, theta, q_range, kv_range):
    import torch

    tdt = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[dtype]
    q, k, v = _inputs((B, S, Hq, D), (B, S, Hk, D), tdt, seed=21)
    scale = 1 / math.sqrt(D)
    out = torch.full((B, S, Hq, D), float("nan"), device=cuda_device)
    lse = torch.full((B, Hq, S), float("nan"), device=cuda_device)
    fa.forward_range(q, k, v, q_range, kv_range, out, lse, softmax_scale=scale, is_causal=causal,
                     rope_theta=theta, out_dtype=torch.float32)
    torch.cuda.synchronize()
    fa.check_status()
    ref_o, ref_l = _oracle(q, k, v, causal, scale, theta, q_range=q_range, kv_range=kv_range)
    got_o, got_l = _np(out), _np(lse)
    _check_rows(got_o, got_l, ref_o, ref_l, q_range, dtype == "float32", "forward_range")
    # Rows outside the range are untouched.
    assert np.isnan(got_o[:, :q_range[0]]).all() and np.isnan(got_o[:, q_range[1]:]).all()
    assert np.isnan(got_l[:, :, :q_range[0]]).all() and np.isnan(got_l[:, :, q_range[1]:]).all()


@pytest.mark.parametrize("dtype,D", [("bfloat16", 128), ("float16", 64), ("float32", 64)])
def test_routed_epilogue_fills_owner_slots(fa, cuda_device, dtype, D):
    import torch

    tdt = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[dtype]
    B, S, Hq, Hk = 2, 700, 4, 1
    R, n_own = 256, 3
    q, k, v = _inputs((B, S, Hq, D), (B, S, Hk, D), tdt, seed=22)
    scale = 1 / math.sqrt(D)
    stage_o = torch.full((n_own, B, R, Hq, D), float("nan"), device=cuda_device)
    stage_l = torch.full((n_own, B, Hq, R), float("nan"), device=cuda_device)
    table = torch.tensor([stage_o[o].data_ptr() for o in range(n_own)] +
                         [stage_l[o].data_ptr() for o in range(n_own)], dtype=torch.int64, device=cuda_device)
    q_range, kv_range = (256, 700), (100, 650)
    fa.forward_range(q, k, v, q_range, kv_range, softmax_scale=scale, is_causal=True, rope_theta=1e4,
                     out_dtype=torch.float32, route=table, n_owners=n_own, owner_rows=R)
    torch.cuda.synchronize()
    fa.check_status()
    ref_o, ref_l = _oracle(q, k, v, True, scale, 1e4, q_range=q_range, kv_range=kv_range)
    so, sl = _np(stage_o), _np(stage_l)
    assert np.isnan(so[0]).all() and np.isnan(sl[0]).all(), "owner 0 holds no row of the range"
    got_o = np.full((B, n_own * R, Hq, D), np.nan, np.float32)
    got_l = np.full((B, Hq, n_own * R), np.nan, np.float32)
    for o in range(n_own):
        got_o[:, o * R:(o + 1) * R] = so[o]
        got_l[:, :, o * R:(o + 1) * R] = sl[o]
    _check_rows(got_o[:, :S], got_l[:, :, :S], ref_o, ref_l, q_range, dtype == "float32", "routed")
    assert np.isnan(got_o[:, S:]).all(), "rows past seqlen_q were written"


@pytest.mark.parametrize("out_dtype", ["float32", "bfloat16"])
def test_combine_of_splits_equals_full_attention(fa, cuda_device, out_dtype):
    import torch

    B, S, Hq, Hk, D = 1, 1500, 8, 1, 128
    q, k, v = _inputs((B, S, Hq, D), (B, S, Hk, D), torch.bfloat16, seed=23, amp=0.5)
    scale = 1 / math.sqrt(D)
    bounds = [0, 256, 640, 1100, 1500]
    n = len(bounds) - 1
    parts_o = torch.empty((n, B, S, Hq, D), device=cuda_device)
    parts_l = torch.empty((n, B, Hq, S), device=cuda_device)
    for j in range(n):
        fa.forward_range(q, k, v, (0, S), (bounds[j], bounds[j + 1]), parts_o[j], parts_l[j],
                         softmax_scale=scale, is_causal=True, rope_theta=5e5, out_dtype=torch.float32)
    odt = {"float32": torch.float32, "bfloat16": torch.bfloat16}[out_dtype]
    out = torch.empty((B, S, Hq, D), dtype=odt, device=cuda_device)
    lse = torch.empty((B, Hq, S), device=cuda_device)
    fa.combine(parts_o, parts_l, out, lse)
    full = fa.forward(q, k, v, softmax_scale=scale, is_causal=True, rope_theta=5e5, out_dtype="float32")
    torch.cuda.synchronize()
    fa.check_status()
    ref_o, ref_l = _oracle(q, k, v, True, scale, 5e5)
    if out_dtype == "float32":
        assert_close_16(_np(out), ref_o, "combine")
        assert np.abs(_np(lse) - ref_l).max() <= 1e-3
        # The merged result and the one-pass kernel agree to accumulation order.
        mx, _ = err_stats(_np(out), _np(full))
        assert mx <= 2e-3
    else:
        # bf16 output: half an ulp of bf16 at |O| < 1 on top of the fp32 bar.
        mx, mean = err_stats(_np(out), ref_o)
        assert mx <= 2e-3 + 4e-3 and mean <= 2e-3


# ------------------------------------------------------------- two GPUs
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _splitkv_worker(rank, world, port, shape, out_dir):
    import torch
    import torch.distributed as dist

    from flash_attn_metal_cpp_b200.multi_gpu import SplitKVAttention

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        B, S, Hq, Hk, D = shape
        # Same CPU-generated inputs as the checking process.
        q, k, v = (t.cuda() for t in _inputs((B, S, Hq, D), (B, S, Hk, D), torch.bfloat16, seed=24, amp=0.5,
                                             device="cpu"))
        att = SplitKVAttention(B, S, S, Hq, Hk, D, causal=True)
        scale = 1 / math.sqrt(D)
        outs = []
        for _ in range(3):  # both staging buffers, then the first again
            outs.append(att.forward(q, k, v, scale, rope_theta=5e5, out_dtype=torch.float32).clone())
        torch.cuda.synchronize()
        att.close()
        lo, hi = att.plan.owner_block(rank)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), lo=lo, hi=hi,
                 o0=outs[0].cpu().numpy(), o1=outs[1].cpu().numpy(), o2=outs[2].cpu().numpy())
    finally:
        dist.destroy_process_group()


def _two_gpus():
    import torch

    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
@pytest.mark.parametrize("shape,rows", [
    ((1, 3000, 8, 1, 128), None),                                          # every row checked
    ((1, 65536, 8, 1, 128), [(0, 128), (20000, 20128), (65408, 65536)]),  # long context, MQA
])
def test_splitkv_two_gpus_matches_oracle(tmp_path, shape, rows):
    import torch
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_splitkv_worker, args=(world, _free_port(), shape, str(tmp_path)), nprocs=world, join=True)
    B, S, Hq, Hk, D = shape
    got = np.full((B, S, Hq, D), np.nan, np.float32)
    for r in range(world):
        z = np.load(os.path.join(str(tmp_path), f"r{r}.npz"))
        lo, hi = int(z["lo"]), int(z["hi"])
        assert np.array_equal(z["o0"], z["o2"]), "repeated steps differ"
        assert np.array_equal(z["o0"], z["o1"]), "the two staging buffers give different results"
        got[:, lo:hi] = z["o0"]
    assert np.isfinite(got).all(), "some rows have no owner"
    q, k, v = _inputs((B, S, Hq, D), (B, S, Hk, D), torch.bfloat16, seed=24, amp=0.5, device="cpu")
    scale = 1 / math.sqrt(D)
    for r0, r1 in (rows or [(0, S)]):
        ref_o, _ = _oracle(q, k, v, True, scale, 5e5, q_range=(r0, r1))
        assert_close_16(got[:, r0:r1], ref_o[:, r0:r1], f"rows {r0}:{r1}")


def test_combine_skips_rows_before_each_partial(fa, cuda_device):
    """Split-KV partials computed only from each split's first key (rounded
    down to a tile), stale (NaN) staging before it: the merge with row_begin
    ignores those rows and equals attention over all keys."""
    import torch

    B, S, Hq, Hk, D = 1, 1400, 8, 1, 128
    q, k, v = _inputs((B, S, Hq, D), (B, S, Hk, D), torch.bfloat16, seed=25, amp=0.5)
    scale = 1 / math.sqrt(D)
    bounds = [0, 300, 700, 1100, 1400]
    n = len(bounds) - 1
    parts_o = torch.full((n, B, S, Hq, D), float("nan"), device=cuda_device)
    parts_l = torch.full((n, B, Hq, S), float("nan"), device=cuda_device)
    starts = []
    for j in range(n):
        q0 = bounds[j] // 128 * 128
        starts.append(q0)
        fa.forward_range(q, k, v, (q0, S), (bounds[j], bounds[j + 1]), parts_o[j], parts_l[j],
                         softmax_scale=scale, is_causal=True, rope_theta=5e5, out_dtype=torch.float32)
    out = torch.empty((B, S, Hq, D), device=cuda_device)
    rb = torch.tensor(starts, dtype=torch.int32, device=cuda_device)
    fa.combine(parts_o, parts_l, out, row_begin=rb)
    torch.cuda.synchronize()
    fa.check_status()
    ref_o, _ = _oracle(q, k, v, True, scale, 5e5)
    assert_close_16(_np(out), ref_o, "combine with row_begin")


def test_forward_range_with_window_and_alibi(fa, cuda_device):
    """forward_range takes the same window / ALiBi arguments as forward: a
    partial over a key range with both matches the oracle."""
    import torch

    B, S, Hq, Hk, D = 1, 900, 4, 2, 128
    q, k, v = _inputs((B, S, Hq, D), (B, S, Hk, D), torch.float16, seed=26)
    scale = 1 / math.sqrt(D)
    sl = np.array([0.5, 0.25, 0.125, 0.0625], np.float32)
    out = torch.full((B, S, Hq, D), float("nan"), device=cuda_device)
    lse = torch.full((B, Hq, S), float("nan"), device=cuda_device)
    fa.forward_range(q, k, v, (128, 900), (200, 800), out, lse, softmax_scale=scale, is_causal=True,
                     out_dtype=torch.float32, window_size=(300, -1), alibi_slopes=torch.from_numpy(sl))
    torch.cuda.synchronize()
    fa.check_status()
    ref_o, ref_l = _oracle(q, k, v, True, scale, None, q_range=(128, 900), kv_range=(200, 800), window=(300, -1),
                           alibi_slopes=sl)
    _check_rows(_np(out), _np(lse), ref_o, ref_l, (128, 900), False, "forward_range window+alibi")
