"""K8/V4 quantised-cache attention: the Attention64 split/combine slot.

The K8/V4 cache is ExLlamaV3's ``CacheLayer_quant`` with 8-bit K and 4-bit V,
the reference's MTP draft cache (src/qwasar_runtime/xqa.py:926-961) and the
cache its ``--prefill flash`` rollback reads through the Attention64
split/combine slot, which keeps the split ABI's 15 + 2 argument order
(docs/superpowers/specs/2026-09-11-qwasar-attention-kernel.md:62-74).

Layout (src/qwasar_bench/prefill_flash.py:32-44):
  k_cache int32 [P, 256, 256], v_cache int32 [P, 256, 128] bit-plane words,
  k_scales / v_scales FP16 [P, 256, 32], one per (token, KV head, 32 dims);
the codes live in the rotated domain R = H32 / sqrt(32) and the reader is
x_rot = FP16((c - (2^(b-1) - 0.5)) * (s / 2^(b-1)))
(docs/superpowers/specs/2026-09-08-direct-k8v4-attention-design.md:55-61).

Every function launches on the current stream of the tensors' device and
raises on CPU tensors: there is no fallback.
"""
from __future__ import annotations

import torch

from . import _lib
from .ops import DIM, HEADS, KV_HEADS, PAGE, _contig, _cuda, _dtype_code, _p, _stream, split_workspace

BLOCK = 32
K_BITS, V_BITS = 8, 4
K_WORDS = KV_HEADS * DIM // BLOCK * K_BITS      # 256
V_WORDS = KV_HEADS * DIM // BLOCK * V_BITS      # 128
SCALES = KV_HEADS * DIM // BLOCK                # 32

__all__ = ["hadamard32", "empty_cache", "check_cache", "append", "split", "combine", "attend", "gather",
           "split_workspace"]


def hadamard32(device=None) -> torch.Tensor:
    """R = H32 / sqrt(32) in natural (Sylvester) order, FP32 [32, 32]:
    R[i, j] = (-1)^popcount(i & j) / sqrt(32).  The split and combine
    kernels take it as h32; with exactly this matrix they rotate the
    queries by the fast butterfly."""
    i = torch.arange(BLOCK)
    x = i[:, None] & i[None, :]
    par = torch.zeros_like(x)
    for b in range(5):
        par ^= (x >> b) & 1
    r = torch.where(par == 1, -1.0, 1.0).to(torch.float32) * torch.tensor(1.0 / 32 ** 0.5, dtype=torch.float32)
    return r.to(device) if device is not None else r


def empty_cache(pages: int, device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(k_cache, v_cache, k_scales, v_scales) of `pages` 256-token pages, zeroed."""
    return (torch.zeros(pages, PAGE, K_WORDS, dtype=torch.int32, device=device),
            torch.zeros(pages, PAGE, V_WORDS, dtype=torch.int32, device=device),
            torch.zeros(pages, PAGE, SCALES, dtype=torch.float16, device=device),
            torch.zeros(pages, PAGE, SCALES, dtype=torch.float16, device=device))


def check_cache(k_cache, v_cache, k_scales, v_scales) -> int:
    """Validates the K8/V4 geometry (the checks of prefill_flash.py:32-44);
    returns the page count."""
    P = k_cache.shape[0]
    if tuple(k_cache.shape) != (P, PAGE, K_WORDS) or tuple(v_cache.shape) != (P, PAGE, V_WORDS):
        raise ValueError("Packed cache geometry must match four 256-dimensional K8/V4 heads")
    if tuple(k_scales.shape) != (P, PAGE, SCALES) or k_scales.shape != v_scales.shape:
        raise ValueError("Quantized cache scales have incompatible geometry")
    if k_cache.dtype != torch.int32 or v_cache.dtype != torch.int32:
        raise ValueError("Packed caches must use int32")
    if k_scales.dtype != torch.half or v_scales.dtype != torch.half:
        raise ValueError("Cache scales must use fp16")
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache), ("k_scales", k_scales), ("v_scales", v_scales)):
        _contig(name, t)
    return P


def _check_table(block_table, cache_seqlens):
    if block_table.dtype != torch.int32 or cache_seqlens.dtype != torch.int32:
        raise ValueError("block table and lengths must be int32")
    _contig("block_table", block_table)
    if cache_seqlens.numel() < 1:
        raise ValueError("cache_seqlens must hold one length")


def _check_h32(h32):
    if h32.dtype != torch.float32 or tuple(h32.shape) != (BLOCK, BLOCK) or not h32.is_contiguous():
        raise ValueError("h32 must be a contiguous FP32 [32, 32] rotation")


def append(k, v, cache, block_table, cache_seqlens) -> None:
    """Quantise new rows k, v [S, 4, 256] (FP16/BF16) into the pages at
    logical positions cache_seqlens[0] + s (the length is not advanced)."""
    kc, vc, ks, vs = cache
    dev = _cuda(k, v, kc, vc, ks, vs, block_table, cache_seqlens)
    P = check_cache(kc, vc, ks, vs)
    _check_table(block_table, cache_seqlens)
    if k.dtype != v.dtype or k.shape != v.shape or tuple(k.shape[-2:]) != (KV_HEADS, DIM):
        raise ValueError("k and v must share dtype and shape [S, 4, 256]")
    _contig("k", k)
    _contig("v", v)
    S = k.numel() // (KV_HEADS * DIM)
    lib = _lib.load()
    _lib.check(lib.qwz_k8v4_append(_p(k), _p(v), _p(kc), _p(vc), _p(ks), _p(vs), _p(block_table),
                                   _p(cache_seqlens), block_table.shape[-1], P, S, _dtype_code(k.dtype),
                                   _stream(dev)), "qwz_k8v4_append")


def split(q, cache, block_table, cache_seqlens, partial_o, partial_ml, h32, num_splits: int,
          split_len: int = 0, sm_scale: float = DIM ** -0.5) -> None:
    """The split kernel over the post-append cache (pre-append length in
    cache_seqlens, q [q_len, 24, 256]); rotated partials into the workspace."""
    kc, vc, ks, vs = cache
    dev = _cuda(q, kc, vc, ks, vs, block_table, cache_seqlens, partial_o, partial_ml, h32)
    P = check_cache(kc, vc, ks, vs)
    _check_table(block_table, cache_seqlens)
    _check_h32(h32)
    if q.dim() != 3 or tuple(q.shape[1:]) != (HEADS, DIM):
        raise ValueError("q must be [q_len, 24, 256]")
    _contig("q", q)
    q_len = q.shape[0]
    if partial_o.numel() < q_len * HEADS * num_splits * DIM or partial_ml.numel() < q_len * HEADS * num_splits * 2:
        raise ValueError("workspace too small for num_splits")
    lib = _lib.load()
    _lib.check(lib.qwz_k8v4_split(_p(q), _p(kc), _p(vc), _p(block_table), _p(cache_seqlens), None,
                                  _p(partial_o), _p(partial_ml), _p(ks), _p(vs), _p(h32), split_len,
                                  block_table.shape[-1], num_splits, None, None, None, q_len, P, sm_scale,
                                  _dtype_code(q.dtype), _stream(dev)), "qwz_k8v4_split")


def combine(partial_o, partial_ml, out, h32, num_splits: int) -> None:
    """Merge the rotated partials and restore out [q_len, 24, 256] = R^T O."""
    dev = _cuda(partial_o, partial_ml, out, h32)
    _check_h32(h32)
    if out.dim() != 3 or tuple(out.shape[1:]) != (HEADS, DIM):
        raise ValueError("out must be [q_len, 24, 256]")
    _contig("out", out)
    lib = _lib.load()
    _lib.check(lib.qwz_k8v4_combine(_p(partial_o), _p(partial_ml), _p(out), _p(h32), num_splits, None,
                                    out.shape[0], _dtype_code(out.dtype), _stream(dev)), "qwz_k8v4_combine")


def attend(q, k, v, cache, block_table, cache_seqlens, out, partial_o, partial_ml, h32, num_splits: int,
           sm_scale: float = DIM ** -0.5) -> torch.Tensor:
    """Append the q_len new rows at cache_seqlens[0].., then attention over
    the post-append cache (three launches, no allocation)."""
    append(k, v, cache, block_table, cache_seqlens)
    split(q, cache, block_table, cache_seqlens, partial_o, partial_ml, h32, num_splits, 0, sm_scale)
    combine(partial_o, partial_ml, out, h32, num_splits)
    return out


def gather(words, scales, block_table, length: int, bits: int) -> torch.Tensor:
    """The reader: logical tokens [0, length) of one cache, FP16 [length, 4, 256], rotated domain."""
    dev = _cuda(words, scales, block_table)
    if words.dtype != torch.int32 or scales.dtype != torch.half:
        raise ValueError("words must be int32 and scales fp16")
    _contig("words", words)
    _contig("scales", scales)
    out = torch.empty(length, KV_HEADS, DIM, dtype=torch.float16, device=dev)
    lib = _lib.load()
    _lib.check(lib.qwz_k8v4_gather(_p(words), _p(scales), _p(block_table), block_table.shape[-1],
                                   words.shape[0], length, bits, _p(out), _stream(dev)), "qwz_k8v4_gather")
    return out
