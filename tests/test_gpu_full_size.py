"""GPU parity at the BASELINE sizes: C2 (65,536-token decode), C3 (MTP7
verify at 32,768 and 131,072), C4 (262,144-token decode on one GPU and as
2/4/8 emulated shards) and C5 (six FP8 draft steps over 65,536 + 6 slots).

The small-size tests check every kernel against the CPU oracle over
oracle-written pools.  Here the pools are filled by the library's NVFP4
writer from seeded device-side rows (BF16 N(0,1), four seed-chosen outlier
channels x8, the BASELINE distribution); a seeded sample of those rows is
re-quantised by the oracle writer and must match the pool bytes exactly.
The oracle then dequantises whatever bytes the pool holds and computes the
FP32 softmax on the same device (its lookup tables follow the operands), so
a 262,144-token check takes seconds.  Two size-independent properties ride
along: a repeated call and a different physical page order give
bit-identical outputs.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4, rng
from qwarz_b200 import sharded
from tests.conftest import assert_close_attention

pytestmark = pytest.mark.gpu

PAGE, KV_HEADS, DIM, HEADS = 256, 4, 256, 24
SAMPLE_ROWS = 256


def _rows(gen, n: int, outl, dtype):
    x = torch.randn(n, KV_HEADS, DIM, generator=gen, device=gen.device)
    x[..., outl] *= 8.0
    return x.to(dtype)


def _pool(cuda, pages: int):
    return [torch.zeros(pages, PAGE, KV_HEADS, DIM // 2, dtype=torch.uint8, device=cuda),
            torch.zeros(pages, PAGE, KV_HEADS, DIM // 2, dtype=torch.uint8, device=cuda),
            torch.zeros(pages, PAGE, KV_HEADS, DIM // 16, dtype=torch.float8_e4m3fn, device=cuda),
            torch.zeros(pages, PAGE, KV_HEADS, DIM // 16, dtype=torch.float8_e4m3fn, device=cuda)]


def _fill(cuda, seed: int, tokens: int, pages: int, dtype=torch.bfloat16):
    """`tokens` seeded rows written by qwz_nvfp4_append into `pages` pages in
    a seed-permuted order.  Returns (pool, table on the device, the numpy
    table, generator, outlier channels); checks a sample of rows byte-exactly
    against the oracle writer."""
    from qwarz_b200 import ops

    table = rng.permutation(seed, pages)
    tdev = torch.from_numpy(table).to(cuda)
    pool = _pool(cuda, pages)
    gen = torch.Generator(device=cuda).manual_seed(seed)
    outl = torch.from_numpy(rng.permutation(seed + 7, DIM)[:4].astype(np.int64)).to(cuda)
    sample = np.sort(rng.permutation(seed + 11, tokens)[:SAMPLE_ROWS]) if tokens else np.zeros(0, np.int64)
    kept_k, kept_v = [], []
    chunk = 16384
    for t0 in range(0, tokens, chunk):
        n = min(chunk, tokens - t0)
        k = _rows(gen, n, outl, dtype)
        v = _rows(gen, n, outl, dtype)
        start = torch.tensor([t0], dtype=torch.int32, device=cuda)
        ops.nvfp4_append(k, v, *pool, tdev, start)
        sel = sample[(sample >= t0) & (sample < t0 + n)] - t0
        idx = torch.from_numpy(sel.astype(np.int64)).to(cuda)
        kept_k.append(k[idx].float().cpu().numpy())
        kept_v.append(v[idx].float().cpu().numpy())
    torch.cuda.synchronize()
    if tokens:
        _check_rows(pool, table, sample, np.concatenate(kept_k), np.concatenate(kept_v))
    return pool, tdev, table, gen, outl


def _check_rows(pool, table, positions, k_rows, v_rows):
    """Pool bytes at `positions` equal the oracle writer's bytes of the rows."""
    pos = np.asarray(positions, np.int64)
    phys = torch.from_numpy(table[pos // PAGE].astype(np.int64)).to(pool[0].device)
    off = torch.from_numpy(pos % PAGE).to(pool[0].device)
    for rows, codes, scales, name in ((k_rows, pool[0], pool[2], "K"), (v_rows, pool[1], pool[3], "V")):
        want_c, want_s = nvfp4.quantize_rows(rows)
        got_c = codes[phys, off].cpu().numpy()
        got_s = scales.view(torch.uint8)[phys, off].cpu().numpy()
        np.testing.assert_array_equal(got_c, want_c, err_msg=f"{name} codes")
        np.testing.assert_array_equal(got_s, want_s, err_msg=f"{name} scales")


def _oracle(q, pool, tdev, pre: int):
    """FP32 oracle on the device over the pool's bytes -> numpy [S, 24, 256]."""
    with torch.no_grad():
        ref = oatt.nvfp4_attention(q.float(), *pool, tdev, pre)
    return ref.cpu().numpy()


def _split_combine(q, pool, tdev, pre: int, splits: int):
    """The split ABI launch plus the combine, no append (the rows are in)."""
    from qwarz_b200 import ops

    lens = torch.tensor([pre], dtype=torch.int32, device=q.device)
    po, pml = ops.split_workspace(q.device, q.shape[0], splits)
    out = torch.empty_like(q)
    ops.attn_split(q, pool[0], pool[1], tdev, lens, po, pml, pool[2], pool[3], splits)
    ops.attn_combine(po, pml, out, splits)
    torch.cuda.synchronize()
    return out


def _attend(q, kn, vn, pool, tdev, pre: int, splits: int):
    """qwz_nvfp4_attend: append the q_len new rows, then decode/verify."""
    from qwarz_b200 import _lib, ops

    lens = torch.tensor([pre], dtype=torch.int32, device=q.device)
    po, pml = ops.split_workspace(q.device, q.shape[0], splits)
    out = torch.empty_like(q)
    _lib.device_error(clear=True)
    ops.nvfp4_attend(q, kn, vn, *pool, tdev, lens, out, po, pml, splits)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    return out


def _dtype_name(dtype) -> str:
    return str(dtype).split(".")[-1]


# --------------------------------------------------------------------- C2
def test_c2_decode_65536(cuda):
    """Decode at 65,536 tokens through qwz_nvfp4_attend (the new row is
    written by the decode kernel itself), the default 37 splits; then the
    split ABI over the same pool twice and over a re-ordered copy."""
    from qwarz_b200 import ops

    dtype, tokens = torch.bfloat16, 65536
    pages = tokens // PAGE
    pool, tdev, table, gen, outl = _fill(cuda, 2002, tokens - 1, pages, dtype)
    q = torch.randn(1, HEADS, DIM, generator=gen, device=cuda).to(dtype)
    kn, vn = _rows(gen, 1, outl, dtype), _rows(gen, 1, outl, dtype)
    splits = ops.default_splits(cuda, tokens)
    out = _attend(q, kn, vn, pool, tdev, tokens - 1, splits)
    _check_rows(pool, table, [tokens - 1], kn.float().cpu().numpy(), vn.float().cpu().numpy())
    ref = _oracle(q, pool, tdev, tokens - 1)
    assert_close_attention(out.float().cpu().numpy(), ref, "C2 decode 65,536", _dtype_name(dtype))

    a = _split_combine(q, pool, tdev, tokens - 1, splits)
    b = _split_combine(q, pool, tdev, tokens - 1, splits)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16)), "repeated call differs"
    assert_close_attention(a.float().cpu().numpy(), ref, "C2 split ABI", _dtype_name(dtype))

    # the same logical sequence in another physical page order
    table2 = rng.permutation(2003, pages)
    t2 = torch.from_numpy(table2).to(cuda)
    pool2 = [torch.empty_like(t) for t in pool]
    for src, dst in zip(pool, pool2):
        dst.view(torch.uint8)[t2.long()] = src.view(torch.uint8)[tdev.long()]
    c = _split_combine(q, pool2, t2, tokens - 1, splits)
    assert torch.equal(a.view(torch.int16), c.view(torch.int16)), "page order changed the output"

    for s in (16, 74):
        d = _split_combine(q, pool, tdev, tokens - 1, s)
        assert_close_attention(d.float().cpu().numpy(), ref, f"C2 splits={s}", _dtype_name(dtype))


# --------------------------------------------------------------------- C3
@pytest.mark.parametrize("tokens", [32768, 131072])
def test_c3_verify_q7(cuda, tokens):
    """MTP7 verify: the 7 new rows appended and attended with the causal
    mask inside the window, at the two BASELINE depths."""
    from qwarz_b200 import ops

    dtype, q_len = torch.float16, 7
    pages = tokens // PAGE
    pre = tokens - q_len
    pool, tdev, table, gen, outl = _fill(cuda, 3000 + pages, pre, pages, dtype)
    q = torch.randn(q_len, HEADS, DIM, generator=gen, device=cuda).to(dtype)
    kn, vn = _rows(gen, q_len, outl, dtype), _rows(gen, q_len, outl, dtype)
    out = _attend(q, kn, vn, pool, tdev, pre, ops.default_splits(cuda, tokens, q_len))
    _check_rows(pool, table, np.arange(pre, tokens), kn.float().cpu().numpy(), vn.float().cpu().numpy())
    ref = _oracle(q, pool, tdev, pre)
    assert_close_attention(out.float().cpu().numpy(), ref, f"C3 verify {tokens}", _dtype_name(dtype))
    again = _split_combine(q, pool, tdev, pre, ops.default_splits(cuda, tokens, q_len))
    assert torch.equal(out.view(torch.int16), again.view(torch.int16)), "verify not repeatable"


# --------------------------------------------------------------------- C4
def test_c4_decode_262144_one_gpu_and_emulated_shards(cuda):
    """262,144 tokens: one GPU through qwz_nvfp4_attend, then the same
    sequence split over 2, 4 and 8 emulated ranks (fused shard split with the
    owner appending, NVLink-layout exchange and merge in one cooperative
    launch).  Every rank must match the oracle and agree bit for bit."""
    import ctypes

    from qwarz_b200 import _lib, ops

    dtype, tokens = torch.bfloat16, 262144
    pages = tokens // PAGE
    pre = tokens - 1
    pool, tdev, table, gen, outl = _fill(cuda, 4004, pre, pages, dtype)
    q = torch.randn(1, HEADS, DIM, generator=gen, device=cuda).to(dtype)
    kn, vn = _rows(gen, 1, outl, dtype), _rows(gen, 1, outl, dtype)
    # the shards' pools start from the pre-append pool
    before = [t.clone() for t in pool]
    out = _attend(q, kn, vn, pool, tdev, pre, ops.default_splits(cuda, tokens))
    _check_rows(pool, table, [pre], kn.float().cpu().numpy(), vn.float().cpu().numpy())
    ref = _oracle(q, pool, tdev, pre)
    assert_close_attention(out.float().cpu().numpy(), ref, "C4 one GPU", _dtype_name(dtype))

    lib = _lib.load()
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    for world in (2, 4, 8):
        shards = sharded.shard_pages(pages, world)
        splits = ops.default_splits(cuda, shards[0].tok_span)
        local = []
        for s in shards:
            phys = tdev[s.first_page:s.first_page + s.num_pages].long()
            local.append([t.view(torch.uint8)[phys].contiguous().view(t.dtype) for t in before])
        ltab = torch.arange(shards[0].num_pages, dtype=torch.int32, device=cuda)
        po = torch.empty(world, HEADS, splits, DIM, dtype=torch.float32, device=cuda)
        pml = torch.empty(world, HEADS, splits, 2, dtype=torch.float32, device=cuda)
        bufs = [torch.zeros(lib.qwz_peer_buffer_bytes(world, 1), dtype=torch.uint8, device=cuda)
                for _ in range(world)]
        peers = (ctypes.c_uint64 * world)(*[b.data_ptr() for b in bufs])
        epochs = torch.zeros(world, HEADS, dtype=torch.int32, device=cuda)
        res = torch.empty(world, HEADS, DIM, dtype=dtype, device=cuda)
        _lib.device_error(clear=True)
        for s in shards:
            lp = local[s.rank]
            ops.shard_split(q, kn, vn, lp[0], lp[1], lp[2], lp[3], ltab[:s.num_pages], lens,
                            po[s.rank], pml[s.rank], s.tok_begin, s.tok_span, splits)
        ops.shard_exchange_combine_emulated(po, pml, splits, peers, bufs[0].numel(), epochs, res)
        torch.cuda.synchronize()
        assert _lib.device_error(clear=True) == 0
        for g in range(world):
            assert torch.equal(res[g], res[0]), f"world={world}: rank {g} differs from rank 0"
        assert_close_attention(res[0].float().cpu().view(1, HEADS, DIM).numpy(), ref,
                               f"C4 {world} emulated ranks", _dtype_name(dtype))
        owner = sharded.owner(pre, shards)
        s = shards[owner]
        phys = tdev[s.first_page:s.first_page + s.num_pages].long()
        for got, want in zip(local[owner], pool):
            assert torch.equal(got.view(torch.uint8), want.view(torch.uint8)[phys]), \
                f"world={world}: the owner's pool differs after its append"


# --------------------------------------------------------------------- C5
def test_c5_draft_six_steps_65536(cuda):
    """Six sequential draft steps over a 65,536-row FP8 shadow with
    per-(page, KV head) FP32 scales and 6 preallocated slots, 16 splits: the
    fused step writes slot 65,536 + i and attends [0, 65,537 + i).  The
    store holds the reference's cast E4M3(clamp(x / scale, +-448)).  Then the
    six steps captured in one CUDA graph must replay to the same outputs."""
    from qwarz_b200.draft_attention import DecodeAttention

    base, steps = 65536, 6
    cap = base + steps
    pages = (cap + PAGE - 1) // PAGE
    gen = torch.Generator(device=cuda).manual_seed(5005)
    outl = torch.from_numpy(rng.permutation(5012, DIM)[:4].astype(np.int64)).to(cuda)
    rows_k = _rows(gen, base, outl, torch.float32)
    rows_v = _rows(gen, base, outl, torch.float32)

    def page_scales(rows):
        padded = torch.zeros(pages * PAGE, KV_HEADS, DIM, device=cuda)
        padded[:base] = rows
        amax = padded.view(pages, PAGE, KV_HEADS, DIM).abs().amax(dim=(1, 3))
        return (amax / 448.0).clamp_min(1e-3)

    ks, vs = page_scales(rows_k), page_scales(rows_v)
    ks[-1], vs[-1] = ks[-2], vs[-2]   # the slots' page: the scale of the page before

    def cast(rows, scale, n):
        per_row = scale.repeat_interleave(PAGE, dim=0)[:n, :, None]
        return (rows / per_row).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)

    k8 = torch.zeros(1, cap, KV_HEADS, DIM, dtype=torch.float8_e4m3fn, device=cuda)
    v8 = torch.zeros_like(k8)
    k8[0, :base] = cast(rows_k, ks, base)
    v8[0, :base] = cast(rows_v, vs, base)
    del rows_k, rows_v
    qs = [torch.randn(1, 1, HEADS, DIM, generator=gen, device=cuda).half() for _ in range(steps)]
    kns = [(torch.randn(KV_HEADS, DIM, generator=gen, device=cuda) * 3).half() for _ in range(steps)]
    vns = [(torch.randn(KV_HEADS, DIM, generator=gen, device=cuda) * 3).half() for _ in range(steps)]
    pos = [torch.tensor([base + i], dtype=torch.int32, device=cuda) for i in range(steps)]
    lens = [torch.tensor([base + i + 1], dtype=torch.int32, device=cuda) for i in range(steps)]
    outs = [torch.empty(1, 1, HEADS, DIM, dtype=torch.float16, device=cuda) for _ in range(steps)]
    attn = DecodeAttention(HEADS, KV_HEADS, DIM, cuda, splits=16)
    page = base // PAGE
    for i in range(steps):
        attn.step(qs[i], kns[i], vns[i], k8, v8, pos[i], lens[i], outs[i], ks, vs)
        torch.cuda.synchronize()
        for new, store, sc in ((kns[i], k8, ks), (vns[i], v8, vs)):
            want = nvfp4.fp8_shadow(new.float().cpu().numpy(), sc[page].cpu().numpy()[:, None])
            np.testing.assert_array_equal(store[0, base + i].view(torch.uint8).cpu().numpy(), want,
                                          err_msg=f"slot {base + i}")
        n = base + i + 1
        per_k = ks.repeat_interleave(PAGE, dim=0)[:n, :, None]
        per_v = vs.repeat_interleave(PAGE, dim=0)[:n, :, None]
        kf = nvfp4.e4m3_decode_torch(k8[0, :n]) * per_k
        vf = nvfp4.e4m3_decode_torch(v8[0, :n]) * per_v
        ref = oatt.attention_fp32(qs[i][0, 0][None].float(), kf, vf, DIM ** -0.5, n - 1)
        assert_close_attention(outs[i].float().cpu().view(1, HEADS, DIM).numpy(), ref.cpu().numpy(),
                               f"C5 draft step {i}")
    eager = [o.clone() for o in outs]

    stream = torch.cuda.Stream(cuda)
    stream.wait_stream(torch.cuda.current_stream(cuda))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            attn.step(qs[i], kns[i], vns[i], k8, v8, pos[i], lens[i], outs[i], ks, vs)
    for o in outs:
        o.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for i in range(steps):
        assert torch.equal(outs[i].view(torch.int16), eager[i].view(torch.int16)), f"graph step {i} differs"
    del graph
