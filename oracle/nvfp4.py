"""NVFP4 / FP8 byte-level restatements — TEST INFRASTRUCTURE ONLY (see package doc).

Layouts (reference engine/forward/attention.py:159-167, xqa.py:103-141):
  codes  uint8 [P, page, heads, dim/2]; element d of a row is the low nibble
         of byte d//2 when d is even, the high nibble when d is odd
  scales E4M3 (stored as uint8) [P, page, heads, dim/16]; element d uses d//16
  code   bits 0-2 index {0, .5, 1, 1.5, 2, 3, 4, 6}, bit 3 is the sign
"""
from __future__ import annotations

import numpy as np
import torch

E2M1_MAGNITUDE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
# value of each 4-bit code (xqa.py:110-136).  The reference negates with
# `-magnitude`, which Triton evaluates as 0 - magnitude, so code 8 is +0.0
# (pinned by the golden gather vectors: code 8 times a positive scale is +0).
E2M1_VALUE = np.concatenate([E2M1_MAGNITUDE, np.float32(0.0) - E2M1_MAGNITUDE]).astype(np.float32)
E2M1_VALUE[8] = np.float32(0.0)


# ----------------------------------------------------------------- E4M3 (fn)
def e4m3_decode(b: np.ndarray) -> np.ndarray:
    """float32 value of E4M3 bytes (bias 7, no infinities, S.1111.111 = NaN)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int32)
    sign = np.where(b & 0x80, -1.0, 1.0).astype(np.float32)
    e = (b >> 3) & 0xF
    m = (b & 7).astype(np.float32)
    sub = m * np.float32(2.0 ** -9)
    nrm = (np.float32(1.0) + m / np.float32(8.0)) * np.ldexp(np.float32(1.0), e - 7).astype(np.float32)
    val = np.where(e == 0, sub, nrm).astype(np.float32) * sign
    return np.where((b & 0x7F) == 0x7F, np.float32(np.nan), val).astype(np.float32)


def e4m3_encode_nonneg(s: np.ndarray) -> np.ndarray:
    """E4M3 byte of non-negative finite float32 values.

    Round to nearest, ties to even; values >= 448 saturate to 448 (0x7E);
    0 and NaN give 0.  Quantum of the binade [2^E, 2^(E+1)) is 2^(E-3) for
    E >= -6 and 2^-9 below (subnormals); a count of 16 quanta rolls into the
    next binade through the +n-8 carry.
    """
    s = np.ascontiguousarray(s, dtype=np.float32)
    bits = s.view(np.uint32)
    E = ((bits >> np.uint32(23)) & np.uint32(0xFF)).astype(np.int32) - 127
    qexp = np.where(E < -6, -9, E - 3)
    scale = np.ldexp(np.float32(1.0), -qexp).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        n = np.nan_to_num(np.rint(s * scale), nan=0.0, posinf=0.0).astype(np.int64)
    code = np.where(E < -6, n, ((E + 7) << 3) + n - 8)
    code = np.where(s > 0, code, 0)
    code = np.where(s >= 448.0, 0x7E, code)
    return code.astype(np.uint8)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Signed E4M3 (RNE) of float32 values clamped to +-448, sign kept (also for 0)."""
    x = np.asarray(x, dtype=np.float32)
    c = np.clip(x, -448.0, 448.0).astype(np.float32)
    mag = e4m3_encode_nonneg(np.abs(c))
    return (mag | np.where(np.signbit(c), 0x80, 0).astype(np.uint8)).astype(np.uint8)


# --------------------------------------------------------------------- E2M1
def e2m1_encode(y: np.ndarray) -> np.ndarray:
    """4-bit code of float32 y: RNE onto {0,.5,1,1.5,2,3,4,6}, saturating at 6.

    Ties go to the even mantissa: 0.25->0, 0.75->1, 1.25->1, 1.75->2,
    2.5->2, 3.5->4, 5->4.  A zero magnitude is always code 0 (never -0).
    """
    a = np.abs(np.asarray(y, dtype=np.float32))
    m = np.select(
        [a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    neg = (np.asarray(y) < 0) & (m != 0)
    return (m | np.where(neg, 8, 0).astype(np.uint8)).astype(np.uint8)


# ------------------------------------------------------------------- writer
def quantize_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """NVFP4 quantisation of rows [..., dim] (dim % 16 == 0).

    Per 16-element block: amax = max|x| (x widened to float32 exactly),
    s = amax / 6 (IEEE float32 division), scale = E4M3(s) (RNE, saturating),
    code = E2M1(x / float(scale)) (IEEE float32 division, then RNE);
    scale 0 -> codes 0.  Returns (codes uint8 [..., dim/2], scales uint8
    [..., dim/16]).
    """
    x = np.asarray(x, dtype=np.float32)
    dim = x.shape[-1]
    blk = x.reshape(*x.shape[:-1], dim // 16, 16)
    amax = np.max(np.abs(blk), axis=-1).astype(np.float32)
    s = (amax / np.float32(6.0)).astype(np.float32)
    sbits = e4m3_encode_nonneg(s)
    sd = e4m3_decode(sbits)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = (blk / sd[..., None]).astype(np.float32)
    codes = np.where((sd > 0)[..., None], e2m1_encode(y), 0).astype(np.uint8)
    codes = codes.reshape(*x.shape[:-1], dim)
    packed = (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)
    return packed, sbits


def dequant_rows(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """float32 values of NVFP4 rows: E2M1 value x float32(E4M3 scale)."""
    packed = np.asarray(packed, dtype=np.uint8)
    lo = packed & 0xF
    hi = packed >> 4
    codes = np.stack([lo, hi], axis=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)
    vals = E2M1_VALUE[codes]
    sc = np.repeat(e4m3_decode(scales), 16, axis=-1)
    return (vals * sc).astype(np.float32)


def append(k: np.ndarray, v: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
           k_scales: np.ndarray, v_scales: np.ndarray, block_table: np.ndarray,
           pre_len: int, page: int = 256) -> None:
    """Restates the writer contract of src/qwasar_runtime/xqa.py:356-379 in place.

    k, v [S, heads, dim]; row i goes to page block_table[(pre+i)//page] at
    offset (pre+i) % page.
    """
    S = k.shape[0]
    for i in range(S):
        pos = pre_len + i
        pp = int(block_table[pos // page])
        off = pos % page
        kc, ks = quantize_rows(k[i])
        vc, vs = quantize_rows(v[i])
        k_cache[pp, off] = kc
        v_cache[pp, off] = vc
        k_scales[pp, off] = ks
        v_scales[pp, off] = vs


def gather(packed: np.ndarray, scales: np.ndarray, block_table: np.ndarray,
           seq_lens: np.ndarray, max_tokens: int, page_size: int) -> np.ndarray:
    """Restates `_gather_nvfp4_kernel` (src/qwasar_runtime/xqa.py:73-143).

    Returns FP16 [batch, max_tokens, heads, dim]; positions at or beyond
    seq_lens[b] are left zero (the reference leaves them unwritten).
    """
    batch = seq_lens.shape[0]
    heads = packed.shape[2]
    dim = packed.shape[3] * 2
    out = np.zeros((batch, max_tokens, heads, dim), dtype=np.float16)
    for b in range(batch):
        n = min(int(seq_lens[b]), max_tokens)
        t = np.arange(n)
        pp = block_table[b, t // page_size]
        off = t % page_size
        vals = dequant_rows(packed[pp, off], scales[pp, off])
        out[b, :n] = vals.astype(np.float16)
    return out


# ----------------------------------------------------------------- FP8 cast
def fp8_shadow(x: np.ndarray, scale: float | np.ndarray = 1.0) -> np.ndarray:
    """E4M3 bytes of x / scale clamped to +-448 (engine/forward/draft.py:209-210
    `_fp8` when scale == 1).  x float16/float32; division in float32."""
    x = np.asarray(x, dtype=np.float32)
    y = x if np.all(np.asarray(scale) == 1.0) else (x / np.asarray(scale, dtype=np.float32)).astype(np.float32)
    return e4m3_encode(y)


# -------------------------------------------------------------- torch views
_E2M1_T = torch.from_numpy(E2M1_VALUE)
_E4M3_T = torch.from_numpy(e4m3_decode(np.arange(256, dtype=np.uint8)))


def dequant_rows_torch(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """float32 dequant of uint8 tensors (same arithmetic as dequant_rows).
    The lookup tables follow the operands' device, so the checker can run
    beside the kernels at full size; the arithmetic is one exact product."""
    e2m1 = _E2M1_T.to(packed.device)
    e4m3 = _E4M3_T.to(packed.device)
    lo = (packed & 0xF).long()
    hi = (packed >> 4).long()
    vals = torch.stack([e2m1[lo], e2m1[hi]], dim=-1).flatten(-2)
    sc = e4m3[scales.view(torch.uint8).long()].repeat_interleave(16, dim=-1)
    return vals * sc


def e4m3_decode_torch(b: torch.Tensor) -> torch.Tensor:
    """float32 values of E4M3 bytes (uint8 or float8_e4m3fn), by table lookup."""
    return _E4M3_T.to(b.device)[b.view(torch.uint8).long()]


def gather_logical_torch(packed: torch.Tensor, scales: torch.Tensor, block_table: torch.Tensor,
                         length: int, page: int = 256, chunk_pages: int = 64) -> torch.Tensor:
    """float32 [length, heads, dim] of the first `length` logical tokens."""
    n_pages = (length + page - 1) // page
    scales = scales.view(torch.uint8)
    parts = []
    for p0 in range(0, n_pages, chunk_pages):
        ids = block_table[p0:min(n_pages, p0 + chunk_pages)].long()
        rows = dequant_rows_torch(packed[ids], scales[ids])
        parts.append(rows.flatten(0, 1))
    return torch.cat(parts, dim=0)[:length]
