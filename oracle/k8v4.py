"""K8/V4 quantised-cache restatement — TEST INFRASTRUCTURE ONLY (see package doc).

The K8/V4 cache is ExLlamaV3's ``CacheLayer_quant`` with k_bits 8 and
v_bits 4 (src/qwasar_runtime/xqa.py:926-961 selects it for the MTP draft
cache; src/qwasar_bench/prefill_flash.py:29-44 checks its geometry).  Its
writer and reader are third-party code that is absent from the reference
tree, so this module restates them from what the reference documents:

  geometry   k_cache int32 [P, 256, 256], v_cache int32 [P, 256, 128],
             k_scales / v_scales FP16 [P, 256, 32]       (prefill_flash.py:32-44)
  blocks     codes of 32 values per (token, KV head, 32-dim block), in the
             rotated domain R = H32 / sqrt(32)
             (docs/superpowers/specs/2026-09-08-direct-k8v4-attention-design.md:55,61)
  reader     x_rot = FP16((FP32(c) - (2^(b-1) - 0.5)) * (FP32(s) / 2^(b-1)))
             (same spec :57; the plan's reader gate restates it,
             docs/superpowers/plans/2026-09-08-direct-k8v4-attention.md:69-72)
  attention  Q rotated, K/V in the rotated domain, output restored with R
             (spec :61)

What the documents leave open is fixed here as ExLlamaV3's published cache
quantiser does it (parity unpinned: no reference output exists to check):

  * the bits of a block are stored as b bit planes, word i of a block holding
    bit i of its 32 codes (bit t = element t), the words of block (h, j) at
    (h * 8 + j) * b .. + b - 1 of the token's row; the scale of the block at
    h * 8 + j of the token's scale row;
  * the writer rotates each block with the natural-order fast Walsh-Hadamard
    butterfly in FP32 (five add/subtract stages, then the factor 1/sqrt(32)),
    takes s = FP16(max |x_rot|) (at most 65504) and the code
    c = clamp(floor(x_rot / s * 2^(b-1) + 2^(b-1)), 0, 2^b - 1), the bin whose
    midpoint the reader returns (c = 2^(b-1) when s = 0).

Every float operation below is a single IEEE FP32 operation in a fixed
order, so the CUDA writer can be compared with it bit for bit.
"""
from __future__ import annotations

import numpy as np
import torch

from .attention import attention_fp32

PAGE, KV_HEADS, DIM, BLOCK = 256, 4, 256, 32
BLOCKS = DIM // BLOCK                                   # 8 blocks per head
K_BITS, V_BITS = 8, 4
INV_SQRT32 = np.float32(1.0 / np.sqrt(32.0))
F16_MAX = np.float32(65504.0)


def hadamard32() -> np.ndarray:
    """R = H32 / sqrt(32), natural (Sylvester) order: R[i, j] = (-1)^popcount(i & j) / sqrt(32)."""
    i = np.arange(BLOCK)
    par = np.vectorize(lambda v: bin(v).count("1") & 1)(i[:, None] & i[None, :])
    return np.where(par == 1, -INV_SQRT32, INV_SQRT32).astype(np.float32)


def rotate_butterfly(x: np.ndarray) -> np.ndarray:
    """R x over the last axis (32), as the writer computes it in FP32: stage s
    (1, 2, 4, 8, 16) sets y_i = x_i + x_(i+s) where bit s of i is clear and
    y_i = x_(i-s) - x_i where it is set; then every element times 1/sqrt(32)."""
    y = np.asarray(x, dtype=np.float32).copy()
    idx = np.arange(BLOCK)
    for s in (1, 2, 4, 8, 16):
        partner = y[..., idx ^ s]
        low = (idx & s) == 0
        y = np.where(low, y + partner, partner - y).astype(np.float32)
    return (y * INV_SQRT32).astype(np.float32)


def quantize_blocks(x_rot: np.ndarray, bits: int) -> tuple[np.ndarray, np.ndarray]:
    """Codes (uint8, [..., 32]) and FP16 scales ([...]) of rotated blocks."""
    x_rot = np.asarray(x_rot, dtype=np.float32)
    amax = np.minimum(np.abs(x_rot).max(axis=-1), F16_MAX).astype(np.float32)
    s16 = amax.astype(np.float16)
    s = s16.astype(np.float32)[..., None]
    m = np.float32(1 << (bits - 1))
    with np.errstate(divide="ignore", invalid="ignore"):
        u = (x_rot / s) * m + m
    # NaN codes as 0 and +-inf saturate, as the device's float-to-integer
    # conversion and clamp do
    c = np.clip(np.floor(np.nan_to_num(u, nan=0.0, posinf=np.float32(1e30), neginf=np.float32(-1e30))), 0,
                (1 << bits) - 1)
    c = np.where(s > 0, c, m)
    return c.astype(np.uint8), s16


def pack_planes(codes: np.ndarray, bits: int) -> np.ndarray:
    """uint32 [..., bits]: word i holds bit i of code t at bit position t."""
    c = np.asarray(codes, dtype=np.uint32)
    shifts = np.arange(BLOCK, dtype=np.uint32)
    return np.stack([(((c >> np.uint32(i)) & np.uint32(1)) << shifts).sum(axis=-1, dtype=np.uint64)
                     .astype(np.uint32) for i in range(bits)], axis=-1)


def unpack_planes(words: np.ndarray, bits: int) -> np.ndarray:
    """Codes uint8 [..., 32] of bit-plane words [..., bits]."""
    w = np.asarray(words).astype(np.uint32)
    t = np.arange(BLOCK, dtype=np.uint32)
    c = np.zeros(w.shape[:-1] + (BLOCK,), dtype=np.uint32)
    for i in range(bits):
        c |= ((w[..., i:i + 1] >> t) & np.uint32(1)) << np.uint32(i)
    return c.astype(np.uint8)


def dequant(codes: np.ndarray, scales: np.ndarray, bits: int) -> np.ndarray:
    """The reader: FP16((FP32(c) - (2^(b-1) - 0.5)) * (FP32(s) / 2^(b-1))).
    codes [..., 32], scales FP16 [...] -> FP16 [..., 32] (rotated domain)."""
    m = np.float32(1 << (bits - 1))
    c = np.asarray(codes).astype(np.float32)
    s = np.asarray(scales, dtype=np.float16).astype(np.float32)[..., None]
    return ((c - (m - np.float32(0.5))) * (s / m)).astype(np.float16)


# ------------------------------------------------------------------ cache
def empty_cache(pages: int) -> dict:
    return {
        "k_cache": np.zeros((pages, PAGE, KV_HEADS * BLOCKS * K_BITS), dtype=np.int32),
        "v_cache": np.zeros((pages, PAGE, KV_HEADS * BLOCKS * V_BITS), dtype=np.int32),
        "k_scales": np.zeros((pages, PAGE, KV_HEADS * BLOCKS), dtype=np.float16),
        "v_scales": np.zeros((pages, PAGE, KV_HEADS * BLOCKS), dtype=np.float16),
    }


def quantize_rows(x: np.ndarray, bits: int) -> tuple[np.ndarray, np.ndarray]:
    """Rows [S, 4, 256] (any float) -> words uint32 [S, 4*8*bits], scales FP16 [S, 32]."""
    S = x.shape[0]
    blocks = np.asarray(x, dtype=np.float32).reshape(S, KV_HEADS * BLOCKS, BLOCK)
    codes, scales = quantize_blocks(rotate_butterfly(blocks), bits)
    return pack_planes(codes, bits).reshape(S, KV_HEADS * BLOCKS * bits), scales


def write_rows(cache: dict, k: np.ndarray, v: np.ndarray, block_table: np.ndarray, start: int) -> None:
    """Append rows k, v [S, 4, 256] at logical positions start.. through the table."""
    S = k.shape[0]
    kw, ks = quantize_rows(k, K_BITS)
    vw, vs = quantize_rows(v, V_BITS)
    pos = start + np.arange(S)
    page = np.asarray(block_table)[pos // PAGE]
    row = pos % PAGE
    cache["k_cache"][page, row] = kw.view(np.int32)
    cache["v_cache"][page, row] = vw.view(np.int32)
    cache["k_scales"][page, row] = ks
    cache["v_scales"][page, row] = vs


def gather_rotated(words: np.ndarray, scales: np.ndarray, block_table: np.ndarray, length: int,
                   bits: int) -> np.ndarray:
    """Logical tokens [0, length) dequantised, rotated domain: FP16 [length, 4, 256]."""
    pos = np.arange(length)
    page = np.asarray(block_table)[pos // PAGE]
    row = pos % PAGE
    w = np.asarray(words)[page, row].view(np.uint32).reshape(length, KV_HEADS * BLOCKS, bits)
    s = np.asarray(scales)[page, row].reshape(length, KV_HEADS * BLOCKS)
    return dequant(unpack_planes(w, bits), s, bits).reshape(length, KV_HEADS, DIM)


def unrotate(x_rot: np.ndarray) -> np.ndarray:
    """R^T x per 32-dim block of the last axis, float64 (R is symmetric and orthogonal)."""
    R = hadamard32().astype(np.float64)
    x = np.asarray(x_rot, dtype=np.float64)
    shp = x.shape
    return (x.reshape(-1, BLOCK) @ R).reshape(shp)


def attention(q: torch.Tensor, cache: dict, block_table: np.ndarray, pre_len: int,
              sm_scale: float = DIM ** -0.5) -> torch.Tensor:
    """FP32 attention over the dequantised cache (post-append, pre_len + S
    tokens), K and V restored from the rotated domain: q [S, 24, 256] ->
    float32 [S, 24, 256].  This is the reference's own oracle shape
    (src/qwasar_bench/prefill_oracle.py:31-52: FP32 softmax attention over the
    dequantised K8/V4 cache, lower-right causal, GQA)."""
    S = q.shape[0]
    L = pre_len + S
    k = unrotate(gather_rotated(cache["k_cache"], cache["k_scales"], block_table, L, K_BITS).astype(np.float32))
    v = unrotate(gather_rotated(cache["v_cache"], cache["v_scales"], block_table, L, V_BITS).astype(np.float32))
    return attention_fp32(q.float().cpu(), torch.from_numpy(k).float(), torch.from_numpy(v).float(), sm_scale,
                          pre_len)


def attention_rotated(q: torch.Tensor, cache: dict, block_table: np.ndarray, pre_len: int,
                      sm_scale: float = DIM ** -0.5) -> torch.Tensor:
    """The same attention computed as the spec describes it (Q rotated, K/V
    left in the rotated domain, the output restored with R); equal to
    `attention` up to FP32 rounding."""
    S = q.shape[0]
    L = pre_len + S
    k = gather_rotated(cache["k_cache"], cache["k_scales"], block_table, L, K_BITS).astype(np.float32)
    v = gather_rotated(cache["v_cache"], cache["v_scales"], block_table, L, V_BITS).astype(np.float32)
    R = hadamard32().astype(np.float64)
    q_rot = (q.double().cpu().numpy().reshape(-1, BLOCK) @ R.T).reshape(q.shape)
    o_rot = attention_fp32(torch.from_numpy(q_rot).float(), torch.from_numpy(k), torch.from_numpy(v), sm_scale,
                           pre_len)
    return torch.from_numpy(unrotate(o_rot.numpy())).float()
