"""Attention forward over the GPUs of one box, one process per GPU.

Two drivers sit on the partitions of `sharding`:

* `unit_forward` -- (batch, KV-head group) shards. Units are independent
  (a query head of group g reads only KV head g, common.metal:215-217), so a
  rank runs the kernel on its shard and no collective touches the data.

* `SplitKVAttention` -- for long sequences with too few heads to fill the
  GPUs (e.g. 8 query heads over one KV head). Keys are split into one
  contiguous range per rank, balanced by visible (query, key) pairs under
  the top-left causal mask; query rows are owned in equal blocks. Each
  rank's kernel computes the partial (O_r, LSE_r) of its keys for the rows
  from its first key on, and its epilogue stores every finished 128-row
  tile straight into the staging slot of the row's owner -- peer memory
  mapped with CUDA IPC, written over NVLink while the rest of the kernel
  still runs. A one-element NCCL all-reduce then orders all partial kernels
  before the owners' merge (fa_combine_ranges: LSE = log sum exp LSE_j,
  O = sum exp(LSE_j - LSE) O_j over the slots written for that row).
  Staging is double-buffered, so the merge of step i and the partial
  stores of step i+1 never touch the same buffer and one barrier per step
  suffices.

No TMA load ever reads peer memory: peers' staging is only written, by the
plain 16-byte stores of the epilogue, and read by nobody but its owner.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _flash_attn_metal as _ext
from . import sharding


class PeerLostError(RuntimeError):
    """A rank of a split-KV group left (or stopped answering) before the merge."""


def merge_barrier(flag: torch.Tensor, group=None) -> None:
    """The one collective of a split-KV step: after it, every rank's partial
    kernel (and its peer stores into the owners' staging) precedes every
    owner's merge in stream order. A peer that exited or never arrives makes
    the backend raise (connection closed, or the process group's timeout);
    that is reported as PeerLostError so no owner merges stale staging."""
    try:
        dist.all_reduce(flag, group=group)
    except Exception as exc:  # gloo: closed connection / timeout; NCCL: communicator error
        raise PeerLostError(f"split-KV merge barrier failed: a peer rank left or did not arrive ({exc})") from exc


class _DeviceArray:
    """Zero-copy torch view of raw device memory (CUDA array interface)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape),
            "typestr": typestr,
            "data": (int(ptr), False),
            "version": 3,
            "strides": None,
        }


def _view(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    typestr = {torch.float32: "<f4", torch.int64: "<i8"}[dtype]
    return torch.as_tensor(_DeviceArray(ptr, shape, typestr), device=device)


class SplitKVAttention:
    """Split-KV attention forward across the ranks of `group` (one GPU each).

    Every rank passes the full Q, K, V (B, S, H, D) CUDA tensors; a rank reads
    only the key range and query rows its share needs. `forward` returns the
    rank's owned block of output rows, (B, rows, Hq, D), rows
    `plan.owner_block(rank)`; ranks >= plan.n_owners get an empty block.
    """

    def __init__(self, batch: int, seqlen_q: int, seqlen_k: int, num_heads_q: int, num_heads_k: int,
                 head_dim: int, causal: bool, group=None, device: Optional[torch.device] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.B, self.Sq, self.Sk = batch, seqlen_q, seqlen_k
        self.Hq, self.Hk, self.D = num_heads_q, num_heads_k, head_dim
        self.causal = causal
        self.plan = sharding.splitkv_plan(seqlen_q, seqlen_k, self.world, causal)
        p = self.plan
        R = p.owner_rows
        # Staging of one owner: world slots of O [B, R, Hq, D] and LSE [B, Hq, R], twice.
        self._o_slot = batch * R * num_heads_q * head_dim * 4
        self._l_slot = batch * num_heads_q * R * 4
        self._o_bytes = self.world * self._o_slot
        self._l_bytes = self.world * self._l_slot
        self._buf_bytes = self._o_bytes + self._l_bytes
        total = 2 * self._buf_bytes
        with torch.cuda.device(self.device):
            self._base, handle = _ext.ipc_alloc(total)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self._peer = []
        with torch.cuda.device(self.device):
            for r in range(self.world):
                self._peer.append(self._base if r == self.rank else _ext.ipc_open(handles[r]))
        # Route tables (one per staging buffer): owner o's O slot and LSE slot of this rank.
        self._routes = []
        for b in range(2):
            tab = [0] * (2 * max(1, p.n_owners))
            for o in range(p.n_owners):
                s = p.slot_of(self.rank, o)
                if s is None:
                    continue
                base = self._peer[o] + b * self._buf_bytes
                tab[o] = base + s * self._o_slot
                tab[p.n_owners + o] = base + self._o_bytes + s * self._l_slot
            self._routes.append(torch.tensor(tab, dtype=torch.int64, device=self.device))
        # Views of this rank's own staging (merged by this rank).
        self._stage = []
        for b in range(2):
            o_ptr = self._base + b * self._buf_bytes
            self._stage.append((
                _view(o_ptr, (self.world, batch, R, num_heads_q, head_dim), torch.float32, self.device),
                _view(o_ptr + self._o_bytes, (self.world, batch, num_heads_q, R), torch.float32, self.device),
            ))
        # Per slot of this rank's block: the first row its rank wrote (a rank's
        # rows start at its first key, so earlier rows of the slot are stale).
        rb = p.row_begin[self.rank] if self.rank < p.n_owners else [0]
        self._row_begin = torch.tensor(rb if rb else [0], dtype=torch.int32, device=self.device)
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._step = 0
        self._closed = False
        dist.barrier(group=group)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, softmax_scale: float,
                cos=None, sin=None, rope_theta: Optional[float] = None, out: Optional[torch.Tensor] = None,
                lse: Optional[torch.Tensor] = None, out_dtype=None, window_size=None,
                alibi_slopes=None) -> torch.Tensor:
        if self._closed:
            raise RuntimeError("SplitKVAttention is closed")
        p = self.plan
        buf = self._step & 1
        self._step += 1
        qlo, qhi = p.q_ranges[self.rank]
        klo, khi = p.kv_ranges[self.rank]
        if qhi > qlo:
            _ext.forward_range(q, k, v, (qlo, qhi), (klo, khi), softmax_scale=softmax_scale,
                               is_causal=self.causal, cos=cos, sin=sin, rope_theta=rope_theta,
                               out_dtype=torch.float32, route=self._routes[buf], n_owners=p.n_owners,
                               owner_rows=p.owner_rows, window_size=window_size, alibi_slopes=alibi_slopes)
        # Every partial kernel precedes every owner's merge (stream-ordered).
        merge_barrier(self._flag, self.group)
        lo, hi = p.owner_block(self.rank)
        rows = hi - lo
        odt = q.dtype if out_dtype is None else out_dtype
        if out is None:
            out = torch.empty((self.B, rows, self.Hq, self.D), dtype=odt, device=q.device)
        if rows > 0:
            n = len(p.slots[self.rank])
            o_st, l_st = self._stage[buf]
            _ext.combine(o_st[:n], l_st[:n], out, lse, q_range=(0, rows), row_begin=self._row_begin[:n])
        return out

    def close(self):
        """Unmap peers' staging and free this rank's (collective: every rank calls it)."""
        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for r, ptr in enumerate(self._peer):
                if r != self.rank:
                    _ext.ipc_close(ptr)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            _ext.ipc_free(self._base)


class QShardAttention:
    """Query-row shards with K/V replicated (the split-KV alternative that
    needs no merge): rank r computes row chunks r and 2W-1-r of 2W against
    every visible key, the two chunks as concurrent launches on two streams.
    No collective touches the data. `forward` writes the rank's rows into a
    (B, Sq, Hq, D) output (of any of the three dtypes) and leaves the other
    rows untouched."""

    def __init__(self, seqlen_q: int, rank: int, world: int, device: Optional[torch.device] = None):
        self.rank, self.world = rank, world
        self.ranges = [r for r in sharding.qshard_ranges(seqlen_q, world)[rank] if r[1] > r[0]]
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self._side = torch.cuda.Stream(self.device)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, softmax_scale: float, causal: bool,
                out: torch.Tensor, cos=None, sin=None, rope_theta: Optional[float] = None, window_size=None,
                alibi_slopes=None) -> torch.Tensor:
        main = torch.cuda.current_stream(self.device)
        kw = dict(softmax_scale=softmax_scale, is_causal=causal, cos=cos, sin=sin, rope_theta=rope_theta,
                  window_size=window_size, alibi_slopes=alibi_slopes, out_dtype=out.dtype)
        Sk = k.shape[1]
        self._side.wait_stream(main)  # inputs written on the main stream are ready
        for i, (lo, hi) in enumerate(self.ranges):
            kv_hi = min(Sk, hi) if causal else Sk  # keys past the chunk's last row are masked
            if i == 0:
                _ext.forward_range(q, k, v, (lo, hi), (0, kv_hi), out, **kw)
            else:
                with torch.cuda.stream(self._side):
                    _ext.forward_range(q, k, v, (lo, hi), (0, kv_hi), out, **kw)
        main.wait_stream(self._side)
        return out


def unit_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rank: int, world: int, **kw) -> torch.Tensor:
    """Rank's (batch, KV-head) shard of the forward: rows of its units, no collective.

    Returns the output of the rank's batch range and query-head range,
    (b_hi - b_lo, Sq, (h_hi - h_lo) * group, D), computed zero-copy on
    strided views of the full tensors.
    """
    B, _, Hq, _ = q.shape
    Hk = k.shape[2]
    g = Hq // Hk
    ranges = sharding.unit_ranges(B, Hk, world, rank)
    if ranges is None:
        raise ValueError("shard of this rank is not a (batch, kv-head) rectangle; use a world that divides B*Hk")
    (b0, b1), (h0, h1) = ranges
    return _ext.forward(q[b0:b1, :, h0 * g:h1 * g], k[b0:b1, :, h0:h1], v[b0:b1, :, h0:h1], **kw)
