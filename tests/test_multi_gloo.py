"""Multi-rank host logic on CPU: world_size-2 gloo ranks run the sharding
plans with the oracle as the compute, exchange results, and must reproduce
the single-process answer. (The GPU path uses the same plans with the CUDA
kernels and one process per GPU.)"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from flash_attn_metal_cpp_b200 import sharding


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs():
    rng = np.random.default_rng(5)
    q = rng.standard_normal((2, 200, 8, 16), dtype=np.float32)
    k = rng.standard_normal((2, 200, 2, 16), dtype=np.float32)
    v = rng.standard_normal((2, 200, 2, 16), dtype=np.float32)
    return q, k, v


def _worker(rank, world, port, mode, result_path):
    import torch
    import torch.distributed as dist

    from oracle import attention_oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, k, v = _inputs()
    B, S, Hq, D = q.shape
    Hk = k.shape[2]
    g = Hq // Hk
    if mode == "units":
        out = np.zeros_like(q)
        for b, hk in sharding.unit_shards(B, Hk, world)[rank]:
            hs = slice(hk * g, (hk + 1) * g)
            out[b:b + 1, :, hs] = orc.attention_ref(q[b:b + 1, :, hs], k[b:b + 1, :, hk:hk + 1],
                                                    v[b:b + 1, :, hk:hk + 1], causal=True, softmax_scale=0.25)
        t = torch.from_numpy(out)
        dist.all_reduce(t)  # disjoint shards: the sum assembles the full output
        result = t.numpy()
    else:  # split-KV: partial (O, LSE) per rank over its zig-zag key chunks, then combine
        parts_o, parts_l = [], []
        for kv in sharding.splitkv_chunks(S, world, align=16)[rank]:
            o, l = orc.attention_ref(q, k, v, causal=True, softmax_scale=0.25, return_lse=True, kv_range=kv)
            parts_o.append(o)
            parts_l.append(l)
        o_all = [torch.zeros(2, *q.shape) for _ in range(world)]
        l_all = [torch.zeros(2, B, Hq, S) for _ in range(world)]
        dist.all_gather(o_all, torch.from_numpy(np.stack(parts_o)))
        dist.all_gather(l_all, torch.from_numpy(np.stack(parts_l)))
        o_cat = torch.cat(o_all).numpy()
        l_cat = torch.cat(l_all).numpy()
        result, _ = orc.combine_partials(o_cat, l_cat)
    if rank == 0:
        np.save(result_path, result)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["units", "splitkv"])
def test_two_rank_plans_reproduce_single_process(tmp_path, mode):
    import torch.multiprocessing as mp

    from oracle import attention_oracle as orc

    path = str(tmp_path / "out.npy")
    mp.spawn(_worker, args=(2, _free_port(), mode, path), nprocs=2, join=True)
    q, k, v = _inputs()
    ref = orc.attention_ref(q, k, v, causal=True, softmax_scale=0.25)
    np.testing.assert_allclose(np.load(path), ref, atol=2e-5)


def test_unit_shards_cover_once():
    for B, H, W in [(4, 8, 1), (4, 8, 2), (4, 8, 8), (1, 8, 8), (3, 5, 4)]:
        shards = sharding.unit_shards(B, H, W)
        flat = [u for s in shards for u in s]
        assert sorted(flat) == [(b, h) for b in range(B) for h in range(H)]
        sizes = [len(s) for s in shards]
        assert max(sizes) - min(sizes) <= 1


def test_zigzag_chunks_balance_causal_work():
    S = 65536
    for W in (2, 4, 8):
        chunks = sharding.splitkv_chunks(S, W)
        flat = sorted(c for r in chunks for c in r)
        assert flat[0][0] == 0 and flat[-1][1] == S
        assert all(a[1] == b[0] for a, b in zip(flat, flat[1:]))
        work = [sum(sharding.causal_work(S, c) for c in r) for r in chunks]
        assert max(work) / min(work) < 1.01
