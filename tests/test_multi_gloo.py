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
    else:  # split-KV: balanced key range per rank, partials routed to row owners' slots, owners merge
        plan = sharding.splitkv_plan(S, S, world, causal=True, tile=16)
        klo, khi = plan.kv_ranges[rank]
        qlo, qhi = plan.q_ranges[rank]
        part_o = np.zeros_like(q)
        part_l = np.full((B, Hq, S), -np.inf, np.float32)
        if qhi > qlo:
            part_o, part_l = orc.attention_ref(q, k, v, causal=True, softmax_scale=0.25, return_lse=True,
                                               kv_range=(klo, khi), q_range=(qlo, qhi))
        # The kernel epilogue stores rows into peers' slots; here the slots are
        # filled from an all_gather of every rank's partial, following the plan.
        o_all = [torch.zeros(*q.shape) for _ in range(world)]
        l_all = [torch.zeros(B, Hq, S) for _ in range(world)]
        dist.all_gather(o_all, torch.from_numpy(np.ascontiguousarray(part_o, dtype=np.float32)))
        dist.all_gather(l_all, torch.from_numpy(np.ascontiguousarray(part_l, dtype=np.float32)))
        block = np.zeros_like(q)
        lo, hi = plan.owner_block(rank)
        if hi > lo:
            slots = plan.slots[rank]
            st_o = np.stack([o_all[r].numpy()[:, lo:hi] for r in slots])
            st_l = np.stack([l_all[r].numpy()[:, :, lo:hi] for r in slots])
            # A slot holds its rank's rows from row_begin on (the rank's first
            # key); earlier rows are stale staging, which the merge skips.
            for j, (r, rb) in enumerate(zip(slots, plan.row_begin[rank])):
                assert plan.q_ranges[r][0] == lo + rb or (rb == 0 and plan.q_ranges[r][0] <= lo)
                st_o[j, :, :rb] = np.nan  # stale
                st_o[j, :, :rb] = 0.0     # ... and skipped
                st_l[j, :, :, :rb] = -np.inf
            block[:, lo:hi], _ = orc.combine_partials(st_o, st_l)
            assert np.isfinite(block[:, lo:hi]).all()
        t = torch.from_numpy(block)
        dist.all_reduce(t)  # owner blocks are disjoint
        result = t.numpy()
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


@pytest.mark.parametrize("Sq,Sk,W,causal", [(65536, 65536, 2, True), (65536, 65536, 8, True), (4096, 4096, 4, True),
                                            (1000, 300, 3, True), (300, 1000, 4, False), (200, 200, 8, True)])
def test_splitkv_plan_covers_and_balances(Sq, Sk, W, causal):
    p = sharding.splitkv_plan(Sq, Sk, W, causal)
    # Key ranges tile [0, Sk) in order.
    assert p.kv_ranges[0][0] == 0 and p.kv_ranges[-1][1] == Sk
    assert all(a[1] == b[0] for a, b in zip(p.kv_ranges, p.kv_ranges[1:]))
    assert all(lo % p.tile == 0 or lo == Sk for lo, _ in p.kv_ranges)
    # Owner blocks tile [0, Sq) with tile-multiple sizes.
    assert p.owner_rows % p.tile == 0 and p.n_owners <= W
    assert p.owner_block(p.n_owners - 1)[1] == Sq
    for r, ((klo, khi), (qlo, qhi)) in enumerate(zip(p.kv_ranges, p.q_ranges)):
        if khi <= klo:
            assert qhi == qlo
            continue
        # Every row that sees a key of the range is computed, starting on an owner boundary.
        first_row = klo if causal else 0
        if first_row < Sq:
            assert qlo <= first_row and qhi == Sq and qlo % p.tile == 0
    # Slots: owner o merges exactly the ranks whose query range reaches into its
    # block, each from the first row that rank wrote.
    for o in range(p.n_owners):
        lo, hi = p.owner_block(o)
        want = [r for r in range(W) if p.q_ranges[r][1] > p.q_ranges[r][0] and p.q_ranges[r][0] < hi
                and p.q_ranges[r][1] > lo]
        assert p.slots[o] == want and len(want) >= 1
        assert p.row_begin[o] == [max(0, p.q_ranges[r][0] - lo) for r in want]
        assert all(0 <= rb < hi - lo for rb in p.row_begin[o])
    for (klo, khi), (qlo, qhi) in zip(p.kv_ranges, p.q_ranges):
        if khi > klo and causal and klo < Sq:
            assert qlo % p.tile == 0 and qlo <= klo < qlo + p.tile  # rows start at the first key's tile
    # Balance: no share exceeds the even share by more than one key tile's work
    # (the granularity of a contiguous tile-aligned cut); long sequences within 5%.
    work = [p.pair_work(r) for r in range(W)]
    tile_max = max(sharding.causal_work(Sq, (t, min(Sk, t + p.tile))) if causal else min(p.tile, Sk - t) * Sq
                   for t in range(0, Sk, p.tile))
    assert max(work) <= sum(work) / W + tile_max
    if Sq >= 65536:
        assert max(work) / min(work) < 1.05


# ------------------------------------------------- a rank leaves before the merge
def _leaver_worker(rank, world, port, how, result_path):
    """Rank 1 leaves before the split-KV merge barrier (it exits, or stays but
    never arrives); rank 0 must get PeerLostError within the process group's
    timeout instead of merging stale staging or waiting forever."""
    import datetime
    import time

    import torch
    import torch.distributed as dist

    from flash_attn_metal_cpp_b200.multi_gpu import PeerLostError, merge_barrier

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
    flag = torch.zeros(1)
    merge_barrier(flag)  # a healthy step: both ranks arrive
    if rank == 1:
        if how == "never_arrives":
            time.sleep(8)  # past rank 0's timeout, then leave without the barrier
        os._exit(0)  # leave between steps, with no collective in flight
    t0 = time.monotonic()
    try:
        merge_barrier(flag)
        outcome = "no error"
    except PeerLostError as exc:
        outcome = "peer lost" if "split-KV merge barrier failed" in str(exc) else f"wrong text: {exc}"
    except Exception as exc:  # noqa: BLE001
        outcome = f"other error: {type(exc).__name__}: {exc}"
    with open(result_path, "w") as f:
        f.write(f"{outcome}\n{time.monotonic() - t0:.2f}\n")
    os._exit(0)  # the group is broken: skip destroy_process_group


@pytest.mark.parametrize("how", ["exits", "never_arrives"])
def test_rank_leaving_before_merge_raises(tmp_path, how):
    import torch.multiprocessing as mp

    path = str(tmp_path / "result.txt")
    ctx = mp.start_processes(_leaver_worker, args=(2, _free_port(), how, path), nprocs=2, join=False,
                             start_method="spawn")
    import time

    deadline = time.monotonic() + 60
    while not ctx.join(timeout=5) and time.monotonic() < deadline:
        pass  # join() returns after each process that ends; wait for both
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    outcome, elapsed = open(path).read().split("\n")[:2]
    assert outcome == "peer lost", outcome
    assert float(elapsed) < 30.0
