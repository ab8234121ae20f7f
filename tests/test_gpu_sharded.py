"""Sequence-sharded decode on one GPU: G shards, each with its own NVFP4 pool
and local block table, reduced to (m, l, O) records by qwz_attn_shard_partial
and merged by qwz_lse_combine_gathered, against the FP32 oracle over the whole
sequence.  (The NCCL exchange between real ranks is the same buffer layout;
its host logic is tested on gloo ranks in test_host.py.)"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4, rng
from qwarz_b200 import sharded
from tests.conftest import assert_close_attention
from tests.golden import cases
from tests.gpu_helpers import make_cache, queries, to_cpu_torch, to_device

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,total", [(2, 2000), (4, 4096), (8, 4100), (3, 1500)])
def test_sharded_records_combine_to_full_attention(cuda, world, total):
    from qwarz_b200 import ops

    pages = (total + 255) // 256 + (1 if world == 8 else 0)
    pages = max(pages, world)
    table = rng.permutation(31 + world, pages)
    c, _, _ = make_cache(500 + world, total, pages, table)
    full = to_cpu_torch(c)
    q = queries(600 + world, 1)
    ref = oatt.nvfp4_attention(q.float(), full["k_cache"], full["v_cache"], full["k_scales"],
                               full["v_scales"], full["table"], total - 1)
    shards = sharded.shard_pages(pages, world)
    gathered = torch.empty(world, 24, 258, dtype=torch.float32, device=cuda)
    lens = torch.tensor([total - 1], dtype=torch.int32, device=cuda)
    qd = q.to(cuda)
    for s in shards:
        # the shard's own pool: its logical pages, physically renumbered 0..n-1
        phys = table[s.first_page:s.first_page + s.num_pages]
        local = {n: np.ascontiguousarray(c[n][phys]) for n in ("k_cache", "v_cache", "k_scales", "v_scales")}
        local["table"] = np.arange(s.num_pages, dtype=np.int32)
        dc = to_device(local, cuda)
        splits = 3
        po, pml = ops.split_workspace(cuda, 1, splits)
        ops.shard_partial(qd, dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"],
                          dc["table"], lens, po, pml, gathered[s.rank], s.tok_begin, s.tok_span, splits)
    out = torch.empty(1, 24, 256, dtype=torch.float16, device=cuda)
    ops.combine_gathered(gathered, out, world)
    torch.cuda.synchronize()
    assert_close_attention(out.float().cpu().numpy(), ref.numpy(), f"sharded world={world}")


def test_shard_append_writes_only_the_owners_rows(cuda):
    """Every shard launches the writer; only the owner of the position stores it."""
    from qwarz_b200 import ops

    world, pages = 2, 4
    shards = sharded.shard_pages(pages, world)
    pre = 2 * 256 + 5          # position owned by rank 1 (pages 2..3)
    k = torch.randn(1, 4, 256, device=cuda).half()
    v = torch.randn(1, 4, 256, device=cuda).half()
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    for s in shards:
        cache = [torch.zeros(s.num_pages, 256, 4, 128, dtype=torch.uint8, device=cuda),
                 torch.zeros(s.num_pages, 256, 4, 128, dtype=torch.uint8, device=cuda),
                 torch.zeros(s.num_pages, 256, 4, 16, dtype=torch.uint8, device=cuda),
                 torch.zeros(s.num_pages, 256, 4, 16, dtype=torch.uint8, device=cuda)]
        table = torch.arange(s.num_pages, dtype=torch.int32, device=cuda)
        ops.nvfp4_append_shard(k, v, *cache, table, lens, s.first_page)
        torch.cuda.synchronize()
        written = any(int(t.count_nonzero()) for t in cache)
        assert written == (s.rank == sharded.owner(pre, shards)), s
    from qwarz_b200 import _lib
    assert _lib.device_error(clear=True) == 0


@pytest.mark.parametrize("world,total,dtype,q_len,pool", [(2, 2000, torch.float16, 1, 0), (3, 1500, torch.float16, 1, 0),
                                                          (4, 4100, torch.bfloat16, 1, 0), (8, 8300, torch.float16, 1, 0),
                                                          (2, 1020, torch.bfloat16, 7, 8), (4, 2044, torch.float16, 7, 16)])
def test_peer_exchange_emulated_ranks_match_full_attention(cuda, world, total, dtype, q_len, pool):
    """Every emulated rank runs the fused shard split (only the owner of a
    new row's page appends it), then all ranks exchange their records through
    peer-layout buffers in one cooperative launch.  Each rank's output must
    match the oracle over the whole sequence and all ranks must agree
    exactly; a second call (the next position) checks that the per-row
    epochs advance; the shard pools must end up holding the oracle's bytes.
    The q_len 7 cases size the pool (`pool` pages) so that the new rows
    cross a shard boundary (token 1024 of 8 pages over 2 ranks, token 2048
    of 16 pages over 4, where the last rank holds no token yet): two ranks
    write rows inside their verify kernels."""
    import ctypes

    from qwarz_b200 import _lib, ops

    lib = _lib.load()
    pages = max((total + 1 + q_len + 255) // 256, world, pool)
    table = rng.permutation(40 + world, pages)
    c, _, _ = make_cache(800 + world, total, pages, table)
    ref = {n: c[n].copy() for n in ("k_cache", "v_cache", "k_scales", "v_scales", "table")}
    shards = sharded.shard_pages(pages, world)
    local = []
    for s in shards:
        phys = table[s.first_page:s.first_page + s.num_pages]
        d = {n: np.ascontiguousarray(c[n][phys]) for n in ("k_cache", "v_cache", "k_scales", "v_scales")}
        d["table"] = np.arange(s.num_pages, dtype=np.int32)
        local.append(to_device(d, cuda))
    rows, splits = 24 * q_len, 3
    po = torch.empty(world, rows, splits, 256, dtype=torch.float32, device=cuda)
    pml = torch.empty(world, rows, splits, 2, dtype=torch.float32, device=cuda)
    bufs = [torch.zeros(lib.qwz_peer_buffer_bytes(world, q_len), dtype=torch.uint8, device=cuda)
            for _ in range(world)]
    peers = (ctypes.c_uint64 * world)(*[b.data_ptr() for b in bufs])
    epochs = torch.zeros(world, rows, dtype=torch.int32, device=cuda)
    out = torch.empty(world, rows, 256, dtype=dtype, device=cuda)
    _lib.device_error(clear=True)
    for step in range(2):
        pre = total + step
        q = queries(900 + 10 * world + step, q_len, dtype)
        kn = torch.from_numpy(cases.kv_rows(950 + step, q_len)).to(dtype)
        vn = torch.from_numpy(cases.kv_rows(960 + step, q_len)).to(dtype)
        nvfp4.append(kn.float().numpy(), vn.float().numpy(), ref["k_cache"], ref["v_cache"], ref["k_scales"],
                      ref["v_scales"], table, pre)
        lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
        qd, kd, vd = q.to(cuda), kn.to(cuda), vn.to(cuda)
        for s in shards:
            dc = local[s.rank]
            ops.shard_split(qd, kd, vd, dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"],
                            dc["table"], lens, po[s.rank], pml[s.rank], s.tok_begin, s.tok_span, splits)
        if q_len == 1:
            ops.shard_exchange_combine_emulated(po, pml, splits, peers, bufs[0].numel(), epochs, out)
        else:
            # rows x world blocks are too many for one cooperative launch at
            # q_len 7: the shards' splits, side by side, are a split set of
            # the whole sequence, which the final combine merges
            po_all = po.permute(1, 0, 2, 3).reshape(rows, world * splits, 256).contiguous()
            pml_all = pml.permute(1, 0, 2, 3).reshape(rows, world * splits, 2).contiguous()
            ops.attn_combine(po_all, pml_all, out[0], world * splits)
            out[1:] = out[0]
        torch.cuda.synchronize()
        expect = oatt.nvfp4_attention(q.float(), **{k: v for k, v in to_cpu_torch(ref).items() if k != "table"},
                                      block_table=torch.from_numpy(table), pre_len=pre)
        for g in range(world):
            assert_close_attention(out[g].float().cpu().view(q_len, 24, 256).numpy(), expect.numpy(),
                                   f"peer exchange world={world} rank={g} step={step}", str(dtype).split(".")[-1])
            assert torch.equal(out[g], out[0]), f"rank {g} differs from rank 0"
    assert (epochs == 2).all() or q_len > 1
    assert _lib.device_error(clear=True) == 0
    for s in shards:
        phys = table[s.first_page:s.first_page + s.num_pages]
        for n in ("k_cache", "v_cache", "k_scales", "v_scales"):
            got = local[s.rank][n].view(torch.uint8).cpu().numpy()
            np.testing.assert_array_equal(got, ref[n][phys], err_msg=f"{n} shard {s.rank}")
