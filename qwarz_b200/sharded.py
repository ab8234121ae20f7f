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

`exchange_records` also runs on gloo CPU tensors, which the host-logic tests
use with oracle-computed records.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops

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


class ShardedDecode:
    """One rank's side of the sharded decode; buffers are allocated once, so
    `step` can be captured in a CUDA graph together with the NCCL call."""

    def __init__(self, shard: Shard, device, q_len: int = 1, num_splits: int | None = None,
                 group=None):
        self.shard = shard
        self.device = torch.device(device)
        self.q_len = q_len
        self.group = group
        self.splits = num_splits or ops.default_splits(self.device, shard.tok_span, q_len)
        self.partial_o, self.partial_ml = ops.split_workspace(self.device, q_len, self.splits)
        rows = q_len * HEADS
        self.send = torch.empty(rows, RECORD, dtype=torch.float32, device=self.device)
        self.gathered = torch.empty(shard.world, rows, RECORD, dtype=torch.float32, device=self.device)

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
        self.append(k, v, cache, local_table, cache_seqlens)
        self.partial(q, cache, local_table, cache_seqlens, sm_scale)
        exchange_records(self.send, self.gathered, self.group)
        ops.combine_gathered(self.gathered, out, self.shard.world)
        return out
