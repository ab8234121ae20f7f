"""Torch-facing wrappers of the C ABI (include/qwz_b200.h).

Each function checks devices, dtypes, shapes and contiguity, then launches on
the current CUDA stream of the tensors' device.  Nothing here synchronises
or allocates (except the convenience `*_workspace` helpers, which must run
before graph capture), and nothing falls back to the CPU: a CPU tensor or a
missing library raises.
"""
from __future__ import annotations

import ctypes

import math

import torch

from . import _lib

HEADS, KV_HEADS, DIM, PAGE = 24, 4, 256, 256
GROUP = HEADS // KV_HEADS
RECORD = DIM + 2  # (m, l, O[256]) per row of a shard partial


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return _lib.DTYPE_F16
    if dt == torch.bfloat16:
        return _lib.DTYPE_BF16
    raise ValueError(f"unsupported activation dtype {dt} (float16 or bfloat16)")


def _cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("qwarz_b200 operators run on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _contig(name: str, t: torch.Tensor) -> None:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def check_cache(k_cache, v_cache, k_scales, v_scales) -> int:
    """Validates the NVFP4 one-level cache geometry; returns the page count."""
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        if t.dtype != torch.uint8 or tuple(t.shape[1:]) != (PAGE, KV_HEADS, DIM // 2):
            raise ValueError(f"{name} must be uint8 [P, 256, 4, 128], got {t.dtype} {tuple(t.shape)}")
        _contig(name, t)
    for name, t in (("k_scales", k_scales), ("v_scales", v_scales)):
        if t.dtype not in (torch.uint8, torch.float8_e4m3fn) or tuple(t.shape[1:]) != (PAGE, KV_HEADS, DIM // 16):
            raise ValueError(f"{name} must be float8_e4m3fn [P, 256, 4, 16], got {t.dtype} {tuple(t.shape)}")
        _contig(name, t)
    P = k_cache.shape[0]
    if v_cache.shape[0] != P or k_scales.shape[0] != P or v_scales.shape[0] != P:
        raise ValueError("caches and scales must have the same page count")
    return P


def _check_lengths(block_table, cache_seqlens):
    if block_table.dtype != torch.int32 or cache_seqlens.dtype != torch.int32:
        raise ValueError("block table and lengths must be int32")
    _contig("block_table", block_table)
    if cache_seqlens.numel() < 1:
        raise ValueError("cache_seqlens must hold one length")


def _check_page_scales(capacity: int, *scales) -> None:
    need = math.ceil(capacity / PAGE) * KV_HEADS
    for s in scales:
        if s is None:
            continue
        if s.dtype != torch.float32 or not s.is_contiguous() or s.numel() < need:
            raise ValueError(f"page scales must be contiguous float32 with >= {need} entries "
                             "([ceil(capacity/256), 4])")


def sm_count(device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def default_splits(device, max_tokens: int, q_len: int = 1) -> int:
    """Splits per KV head: one CTA per SM (decode and verify kernels both
    hold a whole SM), at least one 256-token page per split."""
    pages = max(1, math.ceil(max_tokens / PAGE))
    return int(max(1, min(sm_count(device) // KV_HEADS, pages)))


def split_workspace(device, q_len: int, num_splits: int):
    """(partial_o, partial_ml) for `num_splits` splits (allocate before capture)."""
    rows = q_len * HEADS
    return (torch.empty(rows * num_splits * DIM, dtype=torch.float32, device=device),
            torch.empty(rows * num_splits * 2, dtype=torch.float32, device=device))


# ------------------------------------------------------------------ writers
def nvfp4_append(k, v, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens) -> None:
    """Quantise the new rows k, v [.., S, 4, 256] into the NVFP4 pages at
    positions cache_seqlens[0] + i (reference writer contract, xqa.py:356-379)."""
    dev = _cuda(k, v, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens)
    P = check_cache(k_cache, v_cache, k_scales, v_scales)
    _check_lengths(block_table, cache_seqlens)
    if k.dtype != v.dtype or k.shape != v.shape or k.shape[-2:] != (KV_HEADS, DIM):
        raise ValueError("k and v must share dtype and shape [.., S, 4, 256]")
    _contig("k", k)
    _contig("v", v)
    S = k.numel() // (KV_HEADS * DIM)
    lib = _lib.load()
    _lib.check(lib.qwz_nvfp4_append(
        _p(k), _p(v), _p(k_cache), _p(v_cache), _p(k_scales), _p(v_scales), _p(block_table),
        _p(cache_seqlens), block_table.shape[-1], S, KV_HEADS, PAGE, DIM, P, _dtype_code(k.dtype),
        _stream(dev)), "qwz_nvfp4_append")


def nvfp4_append_shard(k, v, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens,
                       table_page_offset: int) -> None:
    """As nvfp4_append for one shard of a sequence-sharded cache: rows whose
    page is not in this shard's table are skipped."""
    dev = _cuda(k, v, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens)
    P = check_cache(k_cache, v_cache, k_scales, v_scales)
    _check_lengths(block_table, cache_seqlens)
    _contig("k", k)
    _contig("v", v)
    S = k.numel() // (KV_HEADS * DIM)
    lib = _lib.load()
    _lib.check(lib.qwz_nvfp4_append_shard(
        _p(k), _p(v), _p(k_cache), _p(v_cache), _p(k_scales), _p(v_scales), _p(block_table),
        _p(cache_seqlens), block_table.shape[-1], table_page_offset, S, P, _dtype_code(k.dtype),
        _stream(dev)), "qwz_nvfp4_append_shard")


def fp8_shadow_write(k, v, k8, v8, position, k_scale=None, v_scale=None) -> None:
    """Write one new row k, v [.., 4, 256] into the E4M3 shadow at slot position[0]."""
    dev = _cuda(k, v, k8, v8, position, k_scale, v_scale)
    for name, t in (("k8", k8), ("v8", v8)):
        if t.dtype not in (torch.uint8, torch.float8_e4m3fn) or tuple(t.shape[-2:]) != (KV_HEADS, DIM):
            raise ValueError(f"{name} must be E4M3 [.., T, 4, 256]")
        _contig(name, t)
    _contig("k", k)
    _contig("v", v)
    if k.numel() != KV_HEADS * DIM or v.numel() != KV_HEADS * DIM:
        raise ValueError("k and v must hold exactly one row [4, 256]")
    cap = k8.numel() // (KV_HEADS * DIM)
    _check_page_scales(cap, k_scale, v_scale)
    lib = _lib.load()
    _lib.check(lib.qwz_fp8_shadow_write(
        _p(k), _p(v), _p(k8), _p(v8), _p(k_scale), _p(v_scale), _p(position), cap,
        _dtype_code(k.dtype), _stream(dev)), "qwz_fp8_shadow_write")


# ---------------------------------------------------------------- attention
def attn_split(q, k_cache, v_cache, block_table, cache_seqlens, partial_o, partial_ml,
               k_scales, v_scales, num_splits: int, split_len: int = 0,
               sm_scale: float = DIM ** -0.5) -> None:
    """Split ABI launch (partials only); q [.., q_len, 24, 256]."""
    dev = _cuda(q, k_cache, v_cache, block_table, cache_seqlens, partial_o, partial_ml, k_scales, v_scales)
    P = check_cache(k_cache, v_cache, k_scales, v_scales)
    _check_lengths(block_table, cache_seqlens)
    _contig("q", q)
    q_len = q.numel() // (HEADS * DIM)
    lib = _lib.load()
    _lib.check(lib.qwz_attn_split(
        _p(q), _p(k_cache), _p(v_cache), _p(block_table), _p(cache_seqlens), None, _p(partial_o),
        _p(partial_ml), _p(k_scales), _p(v_scales), None, split_len, block_table.shape[-1],
        num_splits, None, None, None, q_len, P, float(sm_scale), _dtype_code(q.dtype),
        _stream(dev)), "qwz_attn_split")


def attn_combine(partial_o, partial_ml, out, num_splits: int) -> None:
    dev = _cuda(partial_o, partial_ml, out)
    _contig("out", out)
    q_len = out.numel() // (HEADS * DIM)
    lib = _lib.load()
    _lib.check(lib.qwz_attn_combine(
        _p(partial_o), _p(partial_ml), _p(out), None, num_splits, None, q_len,
        _dtype_code(out.dtype), _stream(dev)), "qwz_attn_combine")


def nvfp4_attend(q, k, v, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens,
                 out, partial_o, partial_ml, num_splits: int, sm_scale: float = DIM ** -0.5) -> None:
    """Append the q_len new rows, then decode/verify attention into out."""
    dev = _cuda(q, k, v, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens, out,
                partial_o, partial_ml)
    P = check_cache(k_cache, v_cache, k_scales, v_scales)
    _check_lengths(block_table, cache_seqlens)
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        _contig(name, t)
    q_len = q.numel() // (HEADS * DIM)
    if k.numel() != q_len * KV_HEADS * DIM or v.numel() != k.numel():
        raise ValueError("k and v must hold q_len rows [q_len, 4, 256]")
    if out.dtype != q.dtype or out.numel() != q.numel():
        raise ValueError("out must match q")
    if partial_o.numel() < q_len * HEADS * num_splits * DIM or partial_ml.numel() < q_len * HEADS * num_splits * 2:
        raise ValueError("split workspace too small for num_splits")
    lib = _lib.load()
    _lib.check(lib.qwz_nvfp4_attend(
        _p(q), _p(k), _p(v), _p(k_cache), _p(v_cache), _p(k_scales), _p(v_scales),
        _p(block_table), _p(cache_seqlens), _p(out), _p(partial_o), _p(partial_ml),
        block_table.shape[-1], P, q_len, num_splits, float(sm_scale), _dtype_code(q.dtype),
        _stream(dev)), "qwz_nvfp4_attend")


def nvfp4_prefill(q, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens, out,
                  sm_scale: float = DIM ** -0.5) -> None:
    """Prefill attention of q [.., S, 24, 256] over the cache that already
    holds the S new rows (nvfp4_append first): query position s sees keys
    j <= cache_seqlens[0] + s.  Writes out (same shape and type as q)."""
    dev = _cuda(q, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens, out)
    P = check_cache(k_cache, v_cache, k_scales, v_scales)
    _check_lengths(block_table, cache_seqlens)
    _contig("q", q)
    _contig("out", out)
    if out.dtype != q.dtype or out.numel() != q.numel():
        raise ValueError("out must match q")
    S = q.numel() // (HEADS * DIM)
    lib = _lib.load()
    _lib.check(lib.qwz_nvfp4_prefill(
        _p(q), _p(k_cache), _p(v_cache), _p(k_scales), _p(v_scales), _p(block_table),
        _p(cache_seqlens), _p(out), block_table.shape[-1], P, S, float(sm_scale),
        _dtype_code(q.dtype), _stream(dev)), "qwz_nvfp4_prefill")


def draft_prefill(q, k, v, out, sm_scale: float = DIM ** -0.5) -> None:
    """Bottom-right causal attention of q [.., S, 24, 256] FP16 over FP16
    k, v [.., T, 4, 256] (T >= S; head and dim contiguous, any token stride
    that is a multiple of 8): query row s sees keys j <= T - S + s.  Writes
    out (same shape as q)."""
    dev = _cuda(q, k, v, out)
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.dtype != torch.float16:
            raise ValueError(f"{name} must be FP16 (the draft model's dtype)")
    _contig("q", q)
    _contig("out", out)
    if out.numel() != q.numel() or q.shape[-2:] != (HEADS, DIM):
        raise ValueError("q and out must be [.., S, 24, 256]")
    S = q.numel() // (HEADS * DIM)
    rows = []
    for name, t in (("k", k), ("v", v)):
        if t.shape[-2:] != (KV_HEADS, DIM) or t.stride(-1) != 1 or t.stride(-2) != DIM:
            raise ValueError(f"{name} must be [.., T, 4, 256] with head and dim contiguous")
        if any(d != 1 for d in t.shape[:-3]):
            raise ValueError(f"{name} must hold one sequence")
        rows.append((t.shape[-3], t.stride(-3)))
    (T, k_stride), (Tv, v_stride) = rows
    if Tv != T:
        raise ValueError("k and v must have the same number of rows")
    if not 1 <= S <= T:
        raise ValueError("need 1 <= q rows <= k rows (bottom-right causal)")
    lib = _lib.load()
    _lib.check(lib.qwz_draft_prefill(
        _p(q), _p(k), _p(v), _p(out), S, T, k_stride, v_stride, float(sm_scale), _stream(dev)),
        "qwz_draft_prefill")


def shard_partial(q, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens,
                  partial_o, partial_ml, send_buf, tok_begin: int, tok_span: int,
                  num_splits: int, sm_scale: float = DIM ** -0.5) -> None:
    """Local half of the sequence-sharded decode: one (m, l, O) record per row."""
    dev = _cuda(q, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens, partial_o,
                partial_ml, send_buf)
    P = check_cache(k_cache, v_cache, k_scales, v_scales)
    _check_lengths(block_table, cache_seqlens)
    q_len = q.numel() // (HEADS * DIM)
    if send_buf.dtype != torch.float32 or send_buf.numel() < q_len * HEADS * RECORD:
        raise ValueError("send_buf must be float32 with q_len*24*258 elements")
    lib = _lib.load()
    _lib.check(lib.qwz_attn_shard_partial(
        _p(q), _p(k_cache), _p(v_cache), _p(k_scales), _p(v_scales), _p(block_table),
        _p(cache_seqlens), _p(partial_o), _p(partial_ml), _p(send_buf), block_table.shape[-1], P,
        tok_begin, tok_span, q_len, num_splits, float(sm_scale), _dtype_code(q.dtype),
        _stream(dev)), "qwz_attn_shard_partial")


def shard_split(q, k, v, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens,
                partial_o, partial_ml, tok_begin: int, tok_span: int, num_splits: int,
                sm_scale: float = DIM ** -0.5) -> None:
    """Shard split with the new rows appended (only the owning shard stores them)."""
    dev = _cuda(q, k, v, k_cache, v_cache, k_scales, v_scales, block_table, cache_seqlens, partial_o,
                partial_ml)
    P = check_cache(k_cache, v_cache, k_scales, v_scales)
    _check_lengths(block_table, cache_seqlens)
    for name, t in (("q", q), ("k", k), ("v", v)):
        _contig(name, t)
    q_len = q.numel() // (HEADS * DIM)
    if k.numel() != q_len * KV_HEADS * DIM or v.numel() != k.numel():
        raise ValueError("k and v must hold q_len rows [q_len, 4, 256]")
    if partial_o.numel() < q_len * HEADS * num_splits * DIM or partial_ml.numel() < q_len * HEADS * num_splits * 2:
        raise ValueError("split workspace too small for num_splits")
    lib = _lib.load()
    _lib.check(lib.qwz_attn_shard_split(
        _p(q), _p(k), _p(v), _p(k_cache), _p(v_cache), _p(k_scales), _p(v_scales), _p(block_table),
        _p(cache_seqlens), _p(partial_o), _p(partial_ml), block_table.shape[-1], P, tok_begin, tok_span,
        q_len, num_splits, float(sm_scale), _dtype_code(q.dtype), _stream(dev)), "qwz_attn_shard_split")


def shard_exchange_combine(partial_o, partial_ml, num_splits: int, peers, buffer_bytes: int, epochs,
                           rank: int, world: int, out, timeout_ns: int = 0) -> None:
    """Merge this rank's splits, exchange the records over peer memory and merge
    all ranks' records into out; `peers` is a ctypes uint64 array of the
    ranks' exchange buffers as this GPU maps them, `buffer_bytes` the size
    they were allocated with.  The wait for the other ranks gives up after
    timeout_ns (0: 0.5 s) and sets QWZ_DEVERR_TIMEOUT."""
    dev = _cuda(partial_o, partial_ml, epochs, out)
    q_len = out.numel() // (HEADS * DIM)
    if epochs.dtype != torch.int32 or epochs.numel() < q_len * HEADS:
        raise ValueError("epochs must be int32 with q_len*24 elements")
    lib = _lib.load()
    _lib.check(lib.qwz_shard_exchange_combine(
        _p(partial_o), _p(partial_ml), num_splits, q_len, ctypes.cast(peers, ctypes.c_void_p), int(buffer_bytes),
        _p(epochs), rank, world, _p(out), int(timeout_ns), _dtype_code(out.dtype), _stream(dev)),
        "qwz_shard_exchange_combine")


def shard_exchange_combine_emulated(partial_o, partial_ml, num_splits: int, peers, buffer_bytes: int, epochs,
                                    out, timeout_ns: int = 0) -> None:
    """All ranks on one GPU (one cooperative launch): partial_o [world, rows,
    splits, 256], partial_ml [world, rows, splits, 2], epochs int32
    [world, rows], out [world, rows, 256]; peers[g] = rank g's buffer, each
    of buffer_bytes."""
    dev = _cuda(partial_o, partial_ml, epochs, out)
    world = partial_o.shape[0]
    q_len = out[0].numel() // (HEADS * DIM)
    lib = _lib.load()
    _lib.check(lib.qwz_shard_exchange_combine_emulated(
        _p(partial_o), _p(partial_ml), partial_o.shape[2], num_splits, q_len,
        ctypes.cast(peers, ctypes.c_void_p), int(buffer_bytes), _p(epochs), _p(out), world, int(timeout_ns),
        _dtype_code(out.dtype), _stream(dev)), "qwz_shard_exchange_combine_emulated")


def combine_gathered(gathered, out, world: int) -> None:
    dev = _cuda(gathered, out)
    _contig("gathered", gathered)
    q_len = out.numel() // (HEADS * DIM)
    if gathered.dtype != torch.float32 or gathered.numel() < world * q_len * HEADS * RECORD:
        raise ValueError("gathered must be float32 [world, q_len*24, 258]")
    lib = _lib.load()
    _lib.check(lib.qwz_lse_combine_gathered(
        _p(gathered), _p(out), world, q_len, _dtype_code(out.dtype), _stream(dev)),
        "qwz_lse_combine_gathered")


def fp8_draft_decode(q, k8, v8, length, part, stat, out, splits: int, k_scale=None, v_scale=None) -> None:
    dev = _cuda(q, k8, v8, length, part, stat, out, k_scale, v_scale)
    if q.dtype != torch.float16 or out.dtype != torch.float16:
        raise ValueError("draft query and output are float16")
    for name, t in (("q", q), ("k8", k8), ("v8", v8), ("out", out)):
        _contig(name, t)
    cap = k8.numel() // (KV_HEADS * DIM)
    if part.numel() < HEADS * splits * DIM or stat.numel() < HEADS * splits * 2:
        raise ValueError("draft workspace too small for splits")
    _check_page_scales(cap, k_scale, v_scale)
    lib = _lib.load()
    _lib.check(lib.qwz_fp8_draft_decode(
        _p(q), _p(k8), _p(v8), _p(k_scale), _p(v_scale), _p(length), _p(part), _p(stat), _p(out),
        splits, cap, _stream(dev)), "qwz_fp8_draft_decode")


def fp8_draft_step(q, k_new, v_new, position, k8, v8, length, part, stat, out, splits: int,
                   k_scale=None, v_scale=None) -> None:
    """fp8_shadow_write(k_new, v_new, k8, v8, position) then fp8_draft_decode,
    fused: the draft kernel writes the new FP16 rows [4, 256] at slot
    position[0] and attends keys [0, length[0])."""
    dev = _cuda(q, k_new, v_new, position, k8, v8, length, part, stat, out, k_scale, v_scale)
    if q.dtype != torch.float16 or out.dtype != torch.float16:
        raise ValueError("draft query and output are float16")
    for name, t in (("k_new", k_new), ("v_new", v_new)):
        if t.dtype != torch.float16 or t.numel() != KV_HEADS * DIM:
            raise ValueError(f"{name} must be one FP16 row [4, 256]")
        _contig(name, t)
    for name, t in (("q", q), ("k8", k8), ("v8", v8), ("out", out)):
        _contig(name, t)
    for name, t in (("k8", k8), ("v8", v8)):
        if t.dtype not in (torch.uint8, torch.float8_e4m3fn) or tuple(t.shape[-2:]) != (KV_HEADS, DIM):
            raise ValueError(f"{name} must be E4M3 [.., T, 4, 256]")
    cap = k8.numel() // (KV_HEADS * DIM)
    if part.numel() < HEADS * splits * DIM or stat.numel() < HEADS * splits * 2:
        raise ValueError("draft workspace too small for splits")
    _check_page_scales(cap, k_scale, v_scale)
    lib = _lib.load()
    _lib.check(lib.qwz_fp8_draft_step(
        _p(q), _p(k_new), _p(v_new), _p(position), _p(k8), _p(v8), _p(k_scale), _p(v_scale), _p(length),
        _p(part), _p(stat), _p(out), splits, cap, _stream(dev)), "qwz_fp8_draft_step")


def nvfp4_gather(packed, scales, block_table, seq_lens, out, max_tokens: int, page_size: int) -> None:
    """Mirror of the reference `_gather_nvfp4_kernel` launch (xqa.py:73-143)."""
    dev = _cuda(packed, scales, block_table, seq_lens, out)
    for name, t in (("packed", packed), ("scales", scales), ("block_table", block_table), ("out", out)):
        _contig(name, t)
    if out.dtype != torch.float16:
        raise ValueError("gather output is float16")
    batch = seq_lens.numel()
    lib = _lib.load()
    _lib.check(lib.qwz_nvfp4_gather(
        _p(packed), _p(scales), _p(block_table), _p(seq_lens), _p(out), batch, max_tokens,
        block_table.shape[-1], packed.shape[2], packed.shape[3] * 2, page_size, _stream(dev)),
        "qwz_nvfp4_gather")
