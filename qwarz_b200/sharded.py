"""Sequence-page sharding of NVFP4 decode across the GPUs of one node.

New work (the reference is single-GPU; its engine refuses more than one
visible GPU, src/qwasar_runtime/engine.py:602-610).  The logical pages
[0, total) of one sequence are split contiguously: rank g owns pages
[g*total//G, (g+1)*total//G) in its own KV pool, addressed through a local
block table whose entry 0 is its first page.  Q is replicated.  Each call:

  1. append   — every rank launches the writer; only the rank whose shard
                holds position pre + i stores row i (the others skip it);
  2. partial  — split-K attention over the shard, reduced on the device to
                one (m, l, O[256]) FP32 record per query row;
  3. exchange — one all-gather of the records ([G, rows, 258] FP32, about
                24.8 KB per GPU at q_len 1) over NCCL / NVLink;
  4. combine  — every rank LSE-merges the G records in rank order, so the
                output is replicated and identical on all ranks.

With exchange="peer" (the default for NCCL groups on one node) steps 1-2
are one launch (the owning shard appends inside its split kernel) and steps
2b-4 are one kernel over NVLink peer memory (qwz_shard_exchange_combine):
each rank writes its records straight into every rank's exchange buffer
(mapped with CUDA IPC) and merges once all have arrived.

`exchange_records` also runs on gloo CPU tensors, which the host-logic tests
use with oracle-computed records.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib, ops

PAGE = 256
RECORD = ops.RECORD
HEADS = ops.HEADS


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    first_page: int
    num_pages: int

    @property
    def tok_begin(self) -> int:
        return self.first_page * PAGE

    @property
    def tok_span(self) -> int:
        return self.num_pages * PAGE


def shard_pages(total_pages: int, world: int) -> list[Shard]:
    """Contiguous, balanced page ranges; every rank gets at least one page."""
    if world < 1 or total_pages < world:
        raise ValueError(f"cannot shard {total_pages} pages over {world} ranks")
    bounds = [(g * total_pages) // world for g in range(world + 1)]
    return [Shard(g, world, bounds[g], bounds[g + 1] - bounds[g]) for g in range(world)]


def owner(position: int, shards: list[Shard]) -> int:
    """Rank whose shard holds logical token `position`."""
    page = position // PAGE
    for s in shards:
        if s.first_page <= page < s.first_page + s.num_pages:
            return s.rank
    raise ValueError(f"position {position} is outside the sharded sequence")


def exchange_records(send: torch.Tensor, gathered: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather of the per-rank records into gathered [world, ...]."""
    world = dist.get_world_size(group)
    if gathered.shape[0] != world:
        raise ValueError("gathered must have one slot per rank")
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, send.contiguous(), group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), send.contiguous(), group=group)
    return gathered


class PeerExchange:
    """Every rank's exchange buffer mapped on this GPU (CUDA IPC), plus this
    rank's per-row call counters, for qwz_shard_exchange_combine.  Collective:
    every rank of `group` constructs it together."""

    def __init__(self, world: int, rank: int, q_len: int, device, group=None):
        lib = _lib.load()
        self.device = torch.device(device)
        nbytes = lib.qwz_peer_buffer_bytes(world, q_len)
        if nbytes <= 0:
            raise ValueError("world must be 1..8 and q_len 1..8")
        self.nbytes = nbytes
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        with torch.cuda.device(self.device):
            _lib.check(lib.qwz_peer_alloc(nbytes, ctypes.byref(own), handle), "qwz_peer_alloc")
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self._own = own.value
            self._opened = []
            addrs = []
            for g in range(world):
                if g == rank:
                    addrs.append(own.value)
                    continue
                ptr = ctypes.c_void_p()
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(handles[g])
                _lib.check(lib.qwz_peer_open(buf, ctypes.byref(ptr)), "qwz_peer_open")
                self._opened.append(ptr.value)
                addrs.append(ptr.value)
        self.peers = (ctypes.c_uint64 * world)(*addrs)
        self.epochs = torch.zeros(q_len * HEADS, dtype=torch.int32, device=self.device)

    def close(self) -> None:
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                lib.qwz_peer_close(ctypes.c_void_p(ptr))
            self._opened = []
            if self._own:
                lib.qwz_peer_free(ctypes.c_void_p(self._own))
                self._own = None


def _peer_capable(device, world: int, group) -> bool:
    if world < 2 or world > 8 or dist.get_backend(group) != "nccl":
        return False
    here = torch.device(device).index
    n = torch.cuda.device_count()
    return n >= world and all(torch.cuda.can_device_access_peer(here, g) for g in range(n) if g != here)


class ShardedDecode:
    """One rank's side of the sharded decode; buffers are allocated once, so
    `step` can be captured in a CUDA graph (with the NCCL call, or with the
    peer-memory exchange kernel)."""

    def __init__(self, shard: Shard, device, q_len: int = 1, num_splits: int | None = None,
                 group=None, exchange: str = "auto", timeout_ns: int = 0):
        self.shard = shard
        self.timeout_ns = timeout_ns  # bound of the peer exchange's wait (0: 0.5 s)
        self.device = torch.device(device)
        self.q_len = q_len
        self.group = group
        self.splits = num_splits or ops.default_splits(self.device, shard.tok_span, q_len)
        self.partial_o, self.partial_ml = ops.split_workspace(self.device, q_len, self.splits)
        rows = q_len * HEADS
        if exchange == "auto":
            exchange = "peer" if _peer_capable(self.device, shard.world, group) else "nccl"
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'auto', 'peer' or 'nccl'")
        self.exchange = exchange
        self.peer = PeerExchange(shard.world, shard.rank, q_len, self.device, group) if exchange == "peer" else None
        self.send = torch.empty(rows, RECORD, dtype=torch.float32, device=self.device)
        self.gathered = torch.empty(shard.world, rows, RECORD, dtype=torch.float32, device=self.device)

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def append(self, k, v, cache, local_table, cache_seqlens) -> None:
        k_cache, v_cache, k_scales, v_scales = cache
        ops.nvfp4_append_shard(k, v, k_cache, v_cache, k_scales, v_scales, local_table,
                               cache_seqlens, self.shard.first_page)

    def partial(self, q, cache, local_table, cache_seqlens, sm_scale: float = 256 ** -0.5) -> None:
        k_cache, v_cache, k_scales, v_scales = cache
        ops.shard_partial(q, k_cache, v_cache, k_scales, v_scales, local_table, cache_seqlens,
                          self.partial_o, self.partial_ml, self.send, self.shard.tok_begin,
                          self.shard.tok_span, self.splits, sm_scale)

    def step(self, q, k, v, cache, local_table, cache_seqlens, out,
             sm_scale: float = 256 ** -0.5) -> torch.Tensor:
        """Append the new rows, attend over the whole sharded sequence, return out
        (identical on every rank)."""
        if self.peer is not None:
            k_cache, v_cache, k_scales, v_scales = cache
            ops.shard_split(q, k, v, k_cache, v_cache, k_scales, v_scales, local_table, cache_seqlens,
                            self.partial_o, self.partial_ml, self.shard.tok_begin, self.shard.tok_span,
                            self.splits, sm_scale)
            ops.shard_exchange_combine(self.partial_o, self.partial_ml, self.splits, self.peer.peers,
                                       self.peer.nbytes, self.peer.epochs, self.shard.rank, self.shard.world,
                                       out, self.timeout_ns)
            return out
        self.append(k, v, cache, local_table, cache_seqlens)
        self.partial(q, cache, local_table, cache_seqlens, sm_scale)
        exchange_records(self.send, self.gathered, self.group)
        ops.combine_gathered(self.gathered, out, self.shard.world)
        return out
