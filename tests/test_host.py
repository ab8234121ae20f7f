"""Host logic without a GPU: the adapter's contract checks (same messages as
src/qwasar_runtime/xqa.py:307-354), the decline rule, the dispatcher
install, the sequence-shard partition, and the multi-rank exchange + LSE
combine on gloo CPU ranks with oracle-computed shard records, including a
rank that fails."""
from __future__ import annotations

import math
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention as oatt
from oracle import rng
from qwarz_b200 import attention as qattn
from qwarz_b200 import sharded


def _args(**over):
    base = dict(
        bsz=1, q_len=1, num_q_heads=24, dim=256, kv_len=1, num_kv_heads=4,
        q=torch.zeros(1, 1, 24, 256, dtype=torch.float16),
        k=torch.zeros(1, 1, 4, 256, dtype=torch.float16),
        v=torch.zeros(1, 1, 4, 256, dtype=torch.float16),
        k_cache=torch.zeros(2, 256, 4, 128, dtype=torch.uint8),
        v_cache=torch.zeros(2, 256, 4, 128, dtype=torch.uint8),
        causal=True, sm_scale=1 / 16, block_table=torch.zeros(1, 2, dtype=torch.int32),
        cache_seqlens=torch.zeros(1, dtype=torch.int32),
        k_scales=torch.zeros(2, 256, 4, 16, dtype=torch.float8_e4m3fn),
        v_scales=torch.zeros(2, 256, 4, 16, dtype=torch.float8_e4m3fn))
    base.update(over)
    return qattn.AttnArgs(**base)


@pytest.mark.parametrize("over,msg", [
    (dict(bsz=2), "batch size 1"),
    (dict(cu_seqlens=torch.zeros(2)), "varlen"),
    (dict(causal=False), "causal"),
    (dict(window_size=128), "sliding window"),
    (dict(softcap=30.0), "softcap"),
    (dict(q=torch.zeros(1, 1, 24, 256, dtype=torch.float32)), "FP16 queries"),
    (dict(num_q_heads=32), "Q24/KV4/D256"),
    (dict(k_cache=torch.zeros(2, 256, 4, 128, dtype=torch.int8)), "uint8"),
    (dict(k_cache=torch.zeros(2, 128, 4, 128, dtype=torch.uint8)), "cache shape"),
    (dict(v_scales=torch.zeros(2, 256, 4, 8, dtype=torch.float8_e4m3fn)), "scale shape"),
    (dict(block_table=torch.zeros(1, 2, dtype=torch.int64)), "int32"),
    (dict(k=None), "exactly one append"),
    (dict(k=torch.zeros(1, 2, 4, 256, dtype=torch.float16)), "query width"),
    (dict(block_table=torch.zeros(2, 2, dtype=torch.int32)), "batch dimension"),
])
def test_adapter_contract_errors(over, msg):
    adapter = qattn.NVFP4AttentionAdapter()
    with pytest.raises(ValueError, match=msg):
        adapter(_args(**over))


def test_adapter_declines_non_nvfp4():
    assert qattn.NVFP4AttentionAdapter()(_args(k_scales=None)) is None


def test_adapter_valid_args_reach_the_cuda_boundary():
    """Valid CPU tensors pass the contract checks and are refused by the
    operator layer: there is no CPU fallback."""
    with pytest.raises(ValueError, match="CUDA tensors only"):
        qattn.NVFP4AttentionAdapter(decode_graphs=False)(_args())


def test_install_prepends_and_restores():
    fns = ["stock_a", "stock_b"]
    with qattn.install(fns) as runtime:
        assert fns[0] is runtime and fns[1:] == ["stock_a", "stock_b"]
    assert fns == ["stock_a", "stock_b"]


def test_bind_table_pages_and_cache_seqlens():
    t, host = qattn.cache_seqlens(0, "cpu")
    assert host == 0 and t.dtype == torch.int32 and t is qattn.cache_seqlens(0, "cpu")[0]
    t, host = qattn.cache_seqlens(17, "cpu")
    assert host == 17 and t.tolist() == [17]
    dev_len = torch.tensor([5], dtype=torch.int32)
    assert qattn.cache_seqlens(dev_len, "cpu") == (dev_len, None)
    table = qattn._block_table(8, "cpu")
    assert table.tolist() == [list(range(8))]
    cache = qattn.empty_cache(3, "cpu")
    assert [tuple(c.shape) for c in cache] == [(3, 256, 4, 128)] * 2 + [(3, 256, 4, 16)] * 2


# -------------------------------------------------------------- sharding
@pytest.mark.parametrize("pages,world", [(1024, 1), (1024, 2), (1024, 4), (1024, 8), (1000, 3), (9, 8)])
def test_shard_partition_is_contiguous_and_balanced(pages, world):
    shards = sharded.shard_pages(pages, world)
    assert shards[0].first_page == 0
    assert sum(s.num_pages for s in shards) == pages
    for a, b in zip(shards, shards[1:]):
        assert b.first_page == a.first_page + a.num_pages
    sizes = [s.num_pages for s in shards]
    assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1
    for pos in (0, 255, 256, pages * 256 - 1):
        r = sharded.owner(pos, shards)
        assert shards[r].tok_begin <= pos < shards[r].tok_begin + shards[r].tok_span


def test_shard_partition_rejects_too_few_pages():
    with pytest.raises(ValueError):
        sharded.shard_pages(3, 4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_record(q, k, v, begin, end, pre):
    """Oracle (m, l, O) record of one shard in the library's log2 units."""
    L = k.shape[0]
    qg = q.view(1, 4, 6, 256).permute(1, 2, 0, 3).reshape(4, 6, 256)
    kk = k[begin:min(end, L)].permute(1, 0, 2)
    vv = v[begin:min(end, L)].permute(1, 0, 2)
    rec = torch.zeros(24, 258)
    if kk.shape[1] == 0:
        rec[:, 0] = float("-inf")
        return rec
    s = torch.bmm(qg, kk.transpose(1, 2)) / 16 * 1.4426950408889634   # [4, 6, n]
    m = s.max(-1).values
    p = torch.exp2(s - m[..., None])
    rec[:, 0] = m.reshape(24)
    rec[:, 1] = p.sum(-1).reshape(24)
    rec[:, 2:] = torch.bmm(p, vv).reshape(24, 256)
    return rec


def _worker(rank, world, port, total, fail_rank, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        shards = sharded.shard_pages(math.ceil(total / 256), world)
        s = shards[rank]
        q = torch.from_numpy(rng.normal(1, 24 * 256).astype(np.float32)).view(24, 256)
        k = torch.from_numpy(rng.normal(2, total * 1024).astype(np.float32)).view(total, 4, 256)
        v = torch.from_numpy(rng.normal(3, total * 1024).astype(np.float32)).view(total, 4, 256)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the exchange")
        send = _shard_record(q, k, v, s.tok_begin, s.tok_begin + s.tok_span, total - 1)
        gathered = torch.empty(world, 24, 258)
        sharded.exchange_records(send, gathered)
        out = oatt.lse_merge(gathered[:, :, 0], gathered[:, :, 1], gathered[:, :, 2:])
        full = oatt.attention_fp32(q[None], k, v, 1 / 16, total - 1)[0]
        results[rank] = ("ok", float((out - full).abs().max()))
    except Exception as e:  # reported to the parent
        results[rank] = ("error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}")
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world, total, fail_rank=-1):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, fail_rank, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            p.join()
    return dict(results)


@pytest.mark.parametrize("world,total", [(2, 1000), (2, 512), (3, 2000)])
def test_gloo_sharded_exchange_and_combine(world, total):
    res = _run(world, total)
    assert len(res) == world, res
    for r in range(world):
        status, val = res[r]
        assert status == "ok", val
        assert val < 1e-5, (r, val)


def test_gloo_rank_failure_surfaces_as_error_on_peers():
    res = _run(2, 1000, fail_rank=1)
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error", res[0]    # the peer's collective fails (timeout/abort), no hang


def test_bench_algorithmic_bytes_per_layer_call():
    """The roofline's algorithmic bytes: 1,152 B per cached token (codes and
    scales of K and V), Q in and O out, the table, the appended rows and the
    new K/V read, at the BASELINE configs."""
    import bench

    def expect(L, q_len):
        pages = math.ceil(L / 256)
        return 1152 * L + 2 * (q_len * 24 * 256 * 2) + 4 * pages + 1152 * q_len + 2 * q_len * 4 * 256 * 2

    for L, q_len, mb in ((4096, 1, 4.75), (65536, 1, 75.53), (32768, 7, 37.96), (131072, 7, 151.21),
                         (262144, 1, 302.02)):
        got = bench.layer_bytes(L, q_len)
        assert got == expect(L, q_len)
        assert abs(got / 1e6 - mb) < 0.01, (L, q_len, got)


def test_bench_k8v4_token_bytes_follow_the_cache_geometry():
    """The K8/V4 record's algorithmic bytes per token: the bit-plane words of
    K (4 heads x 8 blocks x 8 planes x 4 B) and V (x 4 planes) and the two
    FP16 scale rows (4 x 8 each), as the cache tensors hold them."""
    import bench
    from qwarz_b200 import k8v4

    kc, vc, ks, vs = k8v4.empty_cache(1, "cpu")
    per_token = sum(t[0, 0].numel() * t.element_size() for t in (kc, vc, ks, vs))
    assert per_token == bench.K8V4_TOKEN_BYTES == 1664
