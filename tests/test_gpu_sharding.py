"""The multi-GPU partitions, every rank's share run in turn on one GPU.

* unit_forward: the (batch, KV-head) unit shards of cfg4 (32 units) for
  world sizes 2, 4 and 8 -- each rank's zero-copy strided launch writes its
  own rectangle; together they must cover the output once and equal the
  one-launch forward bit for bit (a unit's CTAs are the same either way).
* QShardAttention: the zig-zag query-row shards of cfg5b (8 query heads over
  one KV head, S = 65536) for world sizes 2, 4 and 8 -- each rank fills its
  two row chunks of one output against every visible key; the union must
  cover every row once and equal the one-launch forward bit for bit.
Both are then compared element by element with the chunked fp32 reference
(gpu_reference.attention_fp32). The split-KV path needs a CUDA IPC mapping
between processes, so it is covered on two GPUs (test_gpu_splitkv.py) and
by bench.py's multi-GPU run.
"""
from __future__ import annotations

import math

import pytest

from conftest import TOL_MAX_ABS_16, TOL_MEAN_ABS_16
from gpu_reference import attention_fp32, compare_whole

pytestmark = pytest.mark.gpu


def _inputs(shape_q, shape_kv, seed, amp, device):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    q = (torch.randn(shape_q, generator=g, device=device) * amp).to(torch.bfloat16)
    k = (torch.randn(shape_kv, generator=g, device=device) * amp).to(torch.bfloat16)
    v = (torch.randn(shape_kv, generator=g, device=device) * amp).to(torch.bfloat16)
    return q, k, v


@pytest.fixture(scope="module")
def cfg4_problem(cuda_device):
    import torch

    import flash_attn_metal_cpp_b200 as pkg

    fa = pkg._flash_attn_metal
    q, k, v = _inputs((4, 8192, 32, 128), (4, 8192, 8, 128), 61, 1.0, cuda_device)
    scale = 1 / math.sqrt(128)
    full = fa.forward(q, k, v, softmax_scale=scale, is_causal=True, rope_theta=5e5, out_dtype="float32")
    ref, _ = attention_fp32(q, k, v, True, scale, 5e5)
    torch.cuda.synchronize()
    return q, k, v, scale, full, ref


@pytest.mark.parametrize("world", [2, 4, 8])
def test_unit_forward_shards_cover_cfg4(cfg4_problem, world):
    import torch

    from flash_attn_metal_cpp_b200 import sharding
    from flash_attn_metal_cpp_b200.multi_gpu import unit_forward

    q, k, v, scale, full, ref = cfg4_problem
    B, _, Hq, _ = q.shape
    Hk = k.shape[2]
    g = Hq // Hk
    out = torch.full_like(full, float("nan"))
    covered = torch.zeros((B, Hq), dtype=torch.int32)
    for rank in range(world):
        part = unit_forward(q, k, v, rank, world, softmax_scale=scale, is_causal=True, rope_theta=5e5,
                            out_dtype="float32")
        (b0, b1), (h0, h1) = sharding.unit_ranges(B, Hk, world, rank)
        assert part.shape == (b1 - b0, q.shape[1], (h1 - h0) * g, q.shape[3])
        out[b0:b1, :, h0 * g:h1 * g] = part
        covered[b0:b1, h0 * g:h1 * g] += 1
    torch.cuda.synchronize()
    assert bool((covered == 1).all()), "unit shards do not cover every (batch, head) exactly once"
    assert torch.equal(out, full), "sharded output differs from the one-launch forward"
    compare_whole(out, ref, TOL_MAX_ABS_16, TOL_MEAN_ABS_16, f"unit shards x{world}")


@pytest.fixture(scope="module")
def cfg5b_problem(cuda_device):
    import torch

    import flash_attn_metal_cpp_b200 as pkg

    fa = pkg._flash_attn_metal
    q, k, v = _inputs((1, 65536, 8, 128), (1, 65536, 1, 128), 62, 0.5, cuda_device)
    scale = 1 / math.sqrt(128)
    full = fa.forward(q, k, v, softmax_scale=scale, is_causal=True, rope_theta=5e5, out_dtype="float32")
    ref, _ = attention_fp32(q, k, v, True, scale, 5e5, row_block=2048)
    torch.cuda.synchronize()
    return q, k, v, scale, full, ref


@pytest.mark.parametrize("world", [2, 4, 8])
def test_qshard_ranks_cover_cfg5b(cfg5b_problem, cuda_device, world):
    import torch

    from flash_attn_metal_cpp_b200.multi_gpu import QShardAttention

    q, k, v, scale, full, ref = cfg5b_problem
    S = q.shape[1]
    out = torch.full_like(full, float("nan"))
    rows = torch.zeros(S, dtype=torch.int32)
    for rank in range(world):
        qs = QShardAttention(S, rank, world, cuda_device)
        qs.forward(q, k, v, scale, True, out, rope_theta=5e5)
        for lo, hi in qs.ranges:
            rows[lo:hi] += 1
    torch.cuda.synchronize()
    assert bool((rows == 1).all()), "query-row shards do not cover every row exactly once"
    assert torch.equal(out, full), "row-sharded output differs from the one-launch forward"
    compare_whole(out, ref, TOL_MAX_ABS_16, TOL_MEAN_ABS_16, f"query-row shards x{world}")
