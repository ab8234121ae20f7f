"""The CUDA-graph routes the engine relies on, and the split ABI called in its
packed argument order.

1. NVFP4AttentionAdapter(decode_graphs=True): the per-(layer, q_len) graph
   that owns append + split + combine (src/qwasar_runtime/xqa.py:156-197,
   440-482, 796-857).  Two eager warm-up calls, a capture, then replays that
   stage q/k/v, the pre-append length and the block table by copy.  Along
   the way the length crosses a page boundary (4093 -> 4097), the table is
   replaced by another and then restored, and a rebuilt scale tensor drops
   the graph (the weak-reference identity check) and leads to a recapture.
   Every call is compared with the same call on an eager adapter over a
   copy of the cache (replay vs eager within 1e-5, the reference's graph
   gate in docs/superpowers/plans/2026-09-11-qwasar-attention-kernel.md:218-220)
   and with the FP32 oracle; the KV and scale bytes of both caches must stay
   identical, and the route counters must show the expected routes.
2. attend() captured inside the caller's graph (as the engine's bucket graph
   captures its forward, engine/forward/resident.py:67-75, 215-266): a
   device cache_len mutated between replays and the table narrowed by
   bind_table_pages.
3. qwz_attn_split / qwz_attn_combine called from pack_split_args output
   (the 15 + 2 argument order of tests/test_attention_kernel_abi.py:13-55).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4, rng
from tests.conftest import assert_close_attention
from tests.gpu_helpers import make_cache, queries, to_cpu_torch, to_device

pytestmark = pytest.mark.gpu

SM = 1 / 16


def _rows(seed, n, dtype, device):
    x = torch.from_numpy(rng.normal(seed, n * 1024).astype(np.float32)).view(1, n, 4, 256)
    return x.to(dtype).to(device)


def _args(dc, q, k, v, lens, table):
    from qwarz_b200.attention import AttnArgs

    S = q.shape[1]
    return AttnArgs(bsz=1, q_len=S, num_q_heads=24, dim=256, kv_len=S, num_kv_heads=4, q=q, k=k, v=v,
                    k_cache=dc["k_cache"], v_cache=dc["v_cache"], causal=True, sm_scale=SM,
                    block_table=table.view(1, -1), cache_seqlens=lens, k_scales=dc["k_scales"],
                    v_scales=dc["v_scales"])


def _cache_bytes(dc):
    return [dc[n].view(torch.uint8).clone() for n in ("k_cache", "v_cache", "k_scales", "v_scales")]


def test_adapter_graph_route_replays_match_eager(cuda):
    from qwarz_b200 import _lib
    from qwarz_b200.attention import NVFP4AttentionAdapter

    pages, pre0 = 20, 4091
    perm_a = rng.permutation(61, pages)
    c, _, _ = make_cache(61, pre0, pages, perm_a)
    dg = to_device(c, cuda)                        # the graph adapter's cache
    de = {n: t.clone() for n, t in dg.items()}     # the eager adapter's cache
    table_a = dg["table"]
    # another table over the same physical pages: same first 16 logical
    # pages (they hold data), the unused tail entries permuted
    perm_b = np.concatenate([perm_a[:16], perm_a[16:][::-1]]).astype(np.int32)
    table_b = torch.from_numpy(perm_b).to(cuda)
    ref = {n: c[n].copy() for n in ("k_cache", "v_cache", "k_scales", "v_scales")}

    ad_g = NVFP4AttentionAdapter(decode_graphs=True)
    ad_e = NVFP4AttentionAdapter(decode_graphs=False)
    # per step: (q_len, table) -- lengths run 4091 .. 4097+, crossing page 16 at 4096
    plan = [(1, "a"), (1, "a"), (1, "a"), (1, "a"), (1, "b"), (1, "b"), (1, "a"),
            ("drop", None), (1, "a"), (1, "a"), (1, "a"), (1, "a"), (7, "a"), (7, "a"), (7, "a"), (7, "a")]
    pos = pre0
    lens = torch.zeros(1, dtype=torch.int32, device=cuda)
    worst = 0.0
    _lib.device_error(clear=True)
    for i, (q_len, tab) in enumerate(plan):
        if q_len == "drop":
            # a rebuilt scale tensor (same bytes, new object): the graph's weak
            # references no longer match, so the adapter drops it
            dg["k_scales"] = dg["k_scales"].clone()
            continue
        table = table_a if tab == "a" else table_b
        phys = perm_a if tab == "a" else perm_b
        q = queries(700 + i, q_len).to(cuda).view(1, q_len, 24, 256)
        k, v = _rows(800 + i, q_len, torch.float16, cuda), _rows(900 + i, q_len, torch.float16, cuda)
        lens.fill_(pos)
        out_g = ad_g(_args(dg, q, k, v, lens, table)).clone()
        out_e = ad_e(_args(de, q, k, v, lens.clone(), table.clone())).clone()
        torch.cuda.synchronize()
        diff = float((out_g.float() - out_e.float()).abs().max())
        worst = max(worst, diff)
        assert diff <= 1e-5, f"step {i}: replay/eager differ by {diff}"
        nvfp4.append(k.float().cpu().numpy()[0], v.float().cpu().numpy()[0], ref["k_cache"], ref["v_cache"],
                     ref["k_scales"], ref["v_scales"], phys, pos)
        expect = oatt.nvfp4_attention(q[0].float().cpu(), *(torch.from_numpy(ref[n]) for n in
                                                             ("k_cache", "v_cache", "k_scales", "v_scales")),
                                      torch.from_numpy(phys), pos, SM)
        assert_close_attention(out_g[0].float().cpu().numpy(), expect.numpy(), f"graph route step {i}")
        pos += q_len
    for a, b, n in zip(_cache_bytes(dg), _cache_bytes(de), ("k_cache", "v_cache", "k_scales", "v_scales")):
        assert torch.equal(a, b), f"{n}: graph and eager caches differ"
        np.testing.assert_array_equal(a.cpu().numpy(), ref[n], err_msg=f"{n} vs the oracle writer")
    assert _lib.device_error(clear=True) == 0
    r = ad_g.diagnostics()["routes"]
    # q_len 1: 2 eager, capture, replays; the drop; 2 eager, capture, replays;
    # q_len 7 (its own graph): 2 eager, capture, replays
    assert r.get("graph_captured") == 3, r
    assert r.get("graph_dropped") == 1, r
    assert r.get("decode_eager") == 6, r
    assert r.get("decode_graph") == len([p for p in plan if p[0] != "drop"]) - 6, r
    assert ad_g.append_calls == len([p for p in plan if p[0] != "drop"])


def test_attend_inside_the_callers_graph(cuda):
    """attend() captured in an outer graph: mutating the device cache_len
    between replays moves the append position and the attended length; the
    table width bound by bind_table_pages is the one captured."""
    from qwarz_b200 import _lib, attention as att, ops

    pages, pre0, bound = 20, 4093, 17
    c, _, _ = make_cache(71, pre0, pages, np.arange(pages, dtype=np.int32))
    dg = to_device(c, cuda)
    de = {n: t.clone() for n, t in dg.items()}
    cache_g = (dg["k_cache"], dg["v_cache"], dg["k_scales"], dg["v_scales"])
    cache_e = (de["k_cache"], de["v_cache"], de["k_scales"], de["v_scales"])
    ref = {n: c[n].copy() for n in ("k_cache", "v_cache", "k_scales", "v_scales")}
    try:
        att.bind_table_pages(bound)
        q = torch.zeros(1, 1, 24, 256, dtype=torch.bfloat16, device=cuda)
        k = torch.zeros(1, 1, 4, 256, dtype=torch.bfloat16, device=cuda)
        v = torch.zeros_like(k)
        cache_len = torch.tensor([pre0], dtype=torch.int32, device=cuda)
        # warm-up outside the capture (the adapter allocates its workspace and
        # output here), on a scratch position that the first step overwrites
        att.attend(q, k, v, cache_g, cache_len)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = att.attend(q, k, v, cache_g, cache_len)
        for i in range(6):  # 4093 .. 4098: crosses into logical page 16
            pos = pre0 + i
            qi = queries(720 + i, 1, torch.bfloat16).to(cuda).view(1, 1, 24, 256)
            ki, vi = _rows(820 + i, 1, torch.bfloat16, cuda), _rows(920 + i, 1, torch.bfloat16, cuda)
            q.copy_(qi)
            k.copy_(ki)
            v.copy_(vi)
            cache_len.fill_(pos)
            graph.replay()
            eager = att.attend(qi, ki, vi, cache_e, pos)
            torch.cuda.synchronize()
            diff = float((out.float() - eager.float()).abs().max())
            assert diff <= 1e-5, f"replay {i}: {diff}"
            nvfp4.append(ki.float().cpu().numpy()[0], vi.float().cpu().numpy()[0], ref["k_cache"], ref["v_cache"],
                         ref["k_scales"], ref["v_scales"], np.arange(pages, dtype=np.int32), pos)
            expect = oatt.nvfp4_attention(qi[0].float().cpu(), *(torch.from_numpy(ref[n]) for n in
                                                                 ("k_cache", "v_cache", "k_scales", "v_scales")),
                                          torch.arange(pages, dtype=torch.int32), pos, 256 ** -0.5)
            assert_close_attention(out[0].float().cpu().numpy(), expect.numpy(), f"outer graph replay {i}",
                                   "bfloat16")
        for n, a, b in zip(("k_cache", "v_cache", "k_scales", "v_scales"), cache_g, cache_e):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)), n
            np.testing.assert_array_equal(a.view(torch.uint8).cpu().numpy(), ref[n], err_msg=n)
        # a position past the bound table is flagged on the device, not written
        _lib.device_error(clear=True)
        cache_len.fill_(bound * 256)
        before = [t.view(torch.uint8).clone() for t in cache_g]
        graph.replay()
        torch.cuda.synchronize()
        assert _lib.device_error(clear=True) & 1, "table-range bit expected past the bound"
        for a, b in zip(before, cache_g):
            assert torch.equal(a, b.view(torch.uint8))
        del graph
    finally:
        att.release_attention_plans()
        att.bind_table_pages(None)


@pytest.mark.parametrize("q_len,split_len,splits", [(1, 0, 20), (1, 512, 8), (7, 0, 11), (7, 1024, 3)])
def test_split_abi_called_with_packed_arguments(cuda, q_len, split_len, splits):
    from qwarz_b200 import _lib, ops
    from qwarz_b200.contract import backend

    pages, pre = 12, 2900
    table = rng.permutation(91, pages)
    c, _, _ = make_cache(91, pre, pages, table)
    dc = to_device(c, cuda)
    full = to_cpu_torch(c)
    q = queries(990 + q_len, q_len).to(cuda)
    k, v = _rows(991, q_len, torch.float16, cuda)[0], _rows(992, q_len, torch.float16, cuda)[0]
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    ops.nvfp4_append(k, v, dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"], dc["table"], lens)
    po, pml = ops.split_workspace(cuda, q_len, splits)
    out = torch.empty_like(q)
    ptrs = {"q": q.data_ptr(), "k_cache": dc["k_cache"].data_ptr(), "v_cache": dc["v_cache"].data_ptr(),
            "block_table": dc["table"].data_ptr(), "cache_seqlens": lens.data_ptr(), "out": out.data_ptr(),
            "partial_o": po.data_ptr(), "partial_ml": pml.data_ptr(), "k_scales": dc["k_scales"].data_ptr(),
            "v_scales": dc["v_scales"].data_ptr()}
    ints = {"split_len": split_len, "num_pages_per_seq": pages, "num_splits": splits}
    packed = backend.pack_split_args(ptrs, ints)
    stream = torch.cuda.current_stream().cuda_stream
    backend.call_split(packed, q_len, pages, SM, _lib.DTYPE_F16, stream)
    backend.call_combine(po.data_ptr(), pml.data_ptr(), out.data_ptr(), splits, q_len, _lib.DTYPE_F16, stream)
    # the same launch through the torch wrappers
    po2, pml2 = ops.split_workspace(cuda, q_len, splits)
    out2 = torch.empty_like(q)
    ops.attn_split(q, dc["k_cache"], dc["v_cache"], dc["table"], lens, po2, pml2, dc["k_scales"], dc["v_scales"],
                   splits, split_len=split_len, sm_scale=SM)
    ops.attn_combine(po2, pml2, out2, splits)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    assert _lib.device_error(clear=True) == 0
    ref = {n: c[n].copy() for n in ("k_cache", "v_cache", "k_scales", "v_scales")}
    nvfp4.append(k.float().cpu().numpy(), v.float().cpu().numpy(), ref["k_cache"], ref["v_cache"],
                 ref["k_scales"], ref["v_scales"], table, pre)
    expect = oatt.nvfp4_attention(q.float().cpu(), *(torch.from_numpy(ref[n]) for n in
                                                     ("k_cache", "v_cache", "k_scales", "v_scales")),
                                  full["table"], pre, SM)
    assert_close_attention(out.float().cpu().numpy(), expect.numpy(), f"packed split q_len={q_len}")


@pytest.mark.parametrize("q_len", [1, 7])
def test_graph_patch_of_split_and_combine_nodes(cuda, q_len):
    """Capture split + combine once, then patch the reference's graph-patch
    indices (split 3, 4, 11, 12, 13 and combine 4) between replays: every
    patched replay must equal eager launches with the same arguments."""
    from qwarz_b200 import _lib, ops
    from qwarz_b200.contract import backend

    pages, pre = 16, 3500
    table_a = rng.permutation(95, pages)
    c, _, _ = make_cache(95, 3800, pages, table_a)
    dc = to_device(c, cuda)
    kc, vc, ks, vs = dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"]
    table_b = torch.from_numpy(rng.permutation(96, pages)).to(cuda)
    q = queries(777, q_len).to(cuda)
    lens_a = torch.tensor([pre], dtype=torch.int32, device=cuda)
    lens_b = torch.tensor([pre + 200 - q_len], dtype=torch.int32, device=cuda)
    po, pml = ops.split_workspace(cuda, q_len, 37)
    out = torch.empty_like(q)

    def launch(table, lens, splits, split_len, o, p_o, p_ml):
        ops.attn_split(q, kc, vc, table, lens, p_o, p_ml, ks, vs, splits, split_len=split_len, sm_scale=SM)
        ops.attn_combine(p_o, p_ml, o, splits)

    def eager(table, lens, splits, split_len):
        o = torch.empty_like(q)
        p_o, p_ml = ops.split_workspace(cuda, q_len, splits)
        launch(table, lens, splits, split_len, o, p_o, p_ml)
        torch.cuda.synchronize()
        return o

    launch(dc["table"], lens_a, 37, 0, out, po, pml)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.graph(g):
        launch(dc["table"], lens_a, 37, 0, out, po, pml)
    g.instantiate()
    graph = g.raw_cuda_graph()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager(dc["table"], lens_a, 37, 0))
    s_nodes = backend.graph_nodes(graph, _lib.NODE_SPLIT)
    c_nodes = backend.graph_nodes(graph, _lib.NODE_COMBINE)
    assert len(s_nodes) == 1 and len(c_nodes) == 1
    width_b = 15
    for table, lens, splits, split_len, exec_too in (
            (table_b, lens_b, 20, 0, True),             # another table, length, split count
            (table_b, lens_b, 8, 512, True),            # fixed 512-token splits
            (dc["table"], lens_a, 37, 0, False)):       # back, patched in the graph only
        ptrs = {"block_table": table.data_ptr(), "cache_seqlens": lens.data_ptr()}
        width = width_b if table is table_b else pages
        packed = backend.pack_split_args(ptrs, {"split_len": split_len, "num_pages_per_seq": width,
                                                "num_splits": splits})
        exe = g.raw_cuda_graph_exec() if exec_too else None
        backend.patch_split(graph, exe, s_nodes[0], packed)
        backend.patch_combine(graph, exe, c_nodes[0], splits)
        if not exec_too:
            g.instantiate()  # a new executable from the patched graph
        g.replay()
        torch.cuda.synchronize()
        expect = eager(table[:width], lens, splits, split_len)
        assert torch.equal(out, expect), (splits, split_len, exec_too)
    assert _lib.device_error(clear=True) == 0
    # the combine node of the sharded merge (another record layout) and a
    # node of another kind are refused
    with pytest.raises(_lib.QwzArgumentError):
        backend.patch_combine(graph, None, s_nodes[0], 4)
    del g
