"""Work partitioning of the attention forward across the GPUs of one box.

The path has no data dependency between (batch, KV-head group) units: every
query head of group g reads only KV head g (common.metal:215-217). Two
partitions follow from that:

* `unit_shards`  -- (batch, KV head) units split into contiguous, equal-size
  blocks per rank; no collective is needed.
* `splitkv_plan` -- for sequences with too few heads to occupy the GPUs,
  the key range is cut into one contiguous range per rank, balanced by the
  number of visible (query, key) pairs under the top-left causal mask. Rank
  r computes partial (O_r, LSE_r) of its keys for every query row at or
  after its first key; query rows are owned in equal blocks, and the
  partial of each row goes to the slot of rank r in its owner's staging
  buffer (written by the kernel epilogue over NVLink). Each owner then
  merges its slots (fa_combine). `splitkv_chunks` is the zig-zag
  alternative (chunks r and 2*world-1-r of 2*world), kept for comparison:
  it balances equally well but gives every rank two partials.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple


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


def qshard_ranges(seqlen_q: int, world: int, align: int = 128) -> List[List[Tuple[int, int]]]:
    """Query-row shards with K/V replicated: rank r takes row chunks r and
    2*world-1-r of 2*world. Under the top-left causal mask the work of a row
    grows linearly with its index, so each pair carries the same work and no
    partial needs merging."""
    return splitkv_chunks(seqlen_q, world, align)


def causal_work(q_rows: int, kv_range: Tuple[int, int]) -> int:
    """Number of visible (query, key) pairs of a key range under the top-left causal mask."""
    lo, hi = kv_range
    total = 0
    for k in range(lo, hi):
        total += max(0, q_rows - k)
    return total


@dataclass
class SplitKVPlan:
    """Split-KV partition of one attention problem over `world` ranks.

    kv_ranges[r]   keys of rank r (contiguous, tile aligned; may be empty)
    q_ranges[r]    query rows rank r computes: from its first visible row
                   (rounded down to a tile) to seqlen_q (all rows without the
                   causal mask); empty when kv_ranges[r] is
    owner_rows     rows per owner block (a multiple of `tile`)
    n_owners       number of owner blocks (ranks >= n_owners own no rows)
    slots[o]       ranks whose partials owner o merges, in slot order
    row_begin[o]   per slot, the first row of owner o's block (block-relative)
                   the slot's rank wrote; the merge ignores the slot before it
    """

    seqlen_q: int
    seqlen_k: int
    world: int
    causal: bool
    tile: int
    owner_rows: int
    n_owners: int
    kv_ranges: List[Tuple[int, int]]
    q_ranges: List[Tuple[int, int]]
    slots: List[List[int]] = field(default_factory=list)
    row_begin: List[List[int]] = field(default_factory=list)

    def owner_block(self, o: int) -> Tuple[int, int]:
        """Query rows [lo, hi) owned by rank o (empty for o >= n_owners)."""
        if o >= self.n_owners:
            return (self.seqlen_q, self.seqlen_q)
        lo = o * self.owner_rows
        return (lo, min(self.seqlen_q, lo + self.owner_rows))

    def slot_of(self, rank: int, owner: int) -> Optional[int]:
        """Slot index of rank's partial in owner's staging buffer (None: not sent)."""
        s = self.slots[owner]
        return s.index(rank) if rank in s else None

    def pair_work(self, rank: int) -> int:
        """Visible (query, key) pairs rank computes."""
        lo, hi = self.kv_ranges[rank]
        if not self.causal:
            return (hi - lo) * self.seqlen_q
        return causal_work(self.seqlen_q, (lo, hi))


def _tile_work(seqlen_q: int, seqlen_k: int, tile: int, causal: bool) -> List[int]:
    """Visible (query, key) pairs per key tile; key k is seen by rows q >= k (top-left)."""
    out = []
    for t in range((seqlen_k + tile - 1) // tile):
        lo, hi = t * tile, min(seqlen_k, (t + 1) * tile)
        if causal:
            # sum_{k=lo}^{hi-1} max(0, Sq - k), closed form over the visible part
            top = min(hi, seqlen_q)
            n = max(0, top - lo)
            out.append(n * seqlen_q - (lo + top - 1) * n // 2 if n else 0)
        else:
            out.append((hi - lo) * seqlen_q)
    return out


def splitkv_plan(seqlen_q: int, seqlen_k: int, world: int, causal: bool, tile: int = 128) -> SplitKVPlan:
    """Balanced contiguous key ranges, owner blocks and slot lists (see SplitKVPlan)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    work = _tile_work(seqlen_q, seqlen_k, tile, causal)
    total = sum(work)
    n_tiles = len(work)
    # Contiguous cut minimising the largest share: the smallest capacity C for
    # which packing tiles in order (a new range whenever C would be exceeded)
    # needs at most `world` ranges (binary search on C).
    def pack(cap):
        cuts, acc = [0], 0
        for t, w in enumerate(work):
            if acc + w > cap and acc > 0:
                cuts.append(t)
                acc = 0
            acc += w
        return cuts

    lo_c, hi_c = max(work, default=0), max(total, 1)
    while lo_c < hi_c:
        mid = (lo_c + hi_c) // 2
        if len(pack(mid)) <= world:
            hi_c = mid
        else:
            lo_c = mid + 1
    bounds = pack(lo_c)
    bounds = bounds + [n_tiles] * (world + 1 - len(bounds))
    kv_ranges = [(min(seqlen_k, bounds[r] * tile), min(seqlen_k, bounds[r + 1] * tile)) for r in range(world)]
    owner_rows = max(tile, -(-seqlen_q // (world * tile)) * tile) if seqlen_q else tile
    n_owners = -(-seqlen_q // owner_rows) if seqlen_q else 0
    q_ranges = []
    for lo, hi in kv_ranges:
        if hi <= lo or seqlen_q == 0:
            q_ranges.append((seqlen_q, seqlen_q))
        elif causal:
            first = min(lo, seqlen_q)  # first row that sees key lo, rounded down to a tile
            q_ranges.append(((first // tile) * tile if first < seqlen_q else seqlen_q, seqlen_q))
        else:
            q_ranges.append((0, seqlen_q))
    slots, row_begin = [], []
    for o in range(n_owners):
        blo = o * owner_rows
        bhi = min(seqlen_q, blo + owner_rows)
        mine = [r for r in range(world) if q_ranges[r][1] > q_ranges[r][0] and q_ranges[r][0] < bhi
                and q_ranges[r][1] > blo]
        slots.append(mine)
        row_begin.append([max(0, q_ranges[r][0] - blo) for r in mine])
    return SplitKVPlan(seqlen_q, seqlen_k, world, causal, tile, owner_rows, n_owners, kv_ranges, q_ranges, slots,
                       row_begin)
