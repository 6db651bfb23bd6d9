"""Work partitioning of the attention forward across the GPUs of one box.

The path has no data dependency between (batch, KV-head group) units: every
query head of group g reads only KV head g (common.metal:215-217). Two
partitions follow from that:

* `unit_shards`  -- (batch, KV head) units split into contiguous, equal-size
  blocks per rank; no collective is needed.
* `splitkv_chunks` -- for sequences with too few heads to occupy the GPUs,
  the key range is cut into 2*world chunks and rank r takes chunks r and
  2*world-1-r ("zig-zag"). Under the top-left causal mask the work of chunk
  c falls linearly with c, so the pairs carry equal work. Each rank produces
  partial (O_j, LSE_j) for its keys; `combine` in the oracle and the
  library's fa_combine merge them.
"""
from __future__ import annotations

from typing import List, Tuple


def unit_shards(batch: int, heads_kv: int, world: int) -> List[List[Tuple[int, int]]]:
    """Units (b, kv_head) of rank r = a contiguous block of the row-major unit list."""
    units = [(b, h) for b in range(batch) for h in range(heads_kv)]
    n = len(units)
    out = []
    for r in range(world):
        lo = (n * r) // world
        hi = (n * (r + 1)) // world
        out.append(units[lo:hi])
    return out


def unit_ranges(batch: int, heads_kv: int, world: int, rank: int):
    """Rank's shard as (batch range, kv-head range) when it is a rectangle, else None."""
    mine = unit_shards(batch, heads_kv, world)[rank]
    if not mine:
        return (0, 0), (0, 0)
    bs = sorted({b for b, _ in mine})
    hs = sorted({h for _, h in mine})
    if len(mine) == len(bs) * len(hs) and bs == list(range(bs[0], bs[-1] + 1)) and hs == list(range(hs[0], hs[-1] + 1)):
        return (bs[0], bs[-1] + 1), (hs[0], hs[-1] + 1)
    return None


def splitkv_chunks(seqlen_k: int, world: int, align: int = 128) -> List[List[Tuple[int, int]]]:
    """Key ranges of each rank: chunks r and 2*world-1-r of 2*world (tile aligned)."""
    n_chunks = 2 * world
    tiles = (seqlen_k + align - 1) // align
    bounds = [min(seqlen_k, ((tiles * c) // n_chunks) * align) for c in range(n_chunks + 1)]
    bounds[-1] = seqlen_k
    chunks = [(bounds[c], bounds[c + 1]) for c in range(n_chunks)]
    return [[chunks[r], chunks[n_chunks - 1 - r]] for r in range(world)]


def causal_work(q_rows: int, kv_range: Tuple[int, int]) -> int:
    """Number of visible (query, key) pairs of a key range under the top-left causal mask."""
    lo, hi = kv_range
    total = 0
    for k in range(lo, hi):
        total += max(0, q_rows - k)
    return total
