"""FP32 attention restatements — TEST INFRASTRUCTURE ONLY (see package doc).

The reference's own oracle for decode/verify is its prefill route
(src/qwasar_runtime/xqa.py:612-673): dequantise the NVFP4 pages to FP16 in
logical order, then SDPA with ``causal_lower_right(q_len, total)``, scale
``sm_scale`` and GQA.  Here the same mask and grouping run in FP32.
"""
from __future__ import annotations

import math

import torch

from . import nvfp4

HEADS, KV_HEADS, DIM, PAGE = 24, 4, 256, 256
GROUP = HEADS // KV_HEADS


def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float,
                   pre_len: int) -> torch.Tensor:
    """q [S, 24, D], k/v [L, 4, D] (L = pre_len + S) -> float32 [S, 24, D].

    Row s of the query sees key j iff j <= pre_len + s (lower-right causal,
    xqa.py:662).  GQA: query head h uses KV head h // 6.
    """
    S = q.shape[0]
    L = k.shape[0]
    qg = q.float().view(S, KV_HEADS, GROUP, DIM).permute(1, 2, 0, 3).reshape(KV_HEADS, GROUP * S, DIM)
    kf = k.float().permute(1, 0, 2)
    vf = v.float().permute(1, 0, 2)
    scores = torch.bmm(qg, kf.transpose(1, 2)) * sm_scale  # [4, 6S, L]
    s_idx = torch.arange(GROUP * S, device=q.device) % S
    visible = torch.arange(L, device=q.device)[None, :] <= (pre_len + s_idx)[:, None]
    scores = scores.masked_fill(~visible[None], float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    out = torch.bmm(probs, vf)  # [4, 6S, D]
    return out.view(KV_HEADS, GROUP, S, DIM).permute(2, 0, 1, 3).reshape(S, HEADS, DIM)


def nvfp4_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    k_scales: torch.Tensor, v_scales: torch.Tensor, block_table: torch.Tensor,
                    pre_len: int, sm_scale: float = DIM ** -0.5) -> torch.Tensor:
    """Decode/verify oracle over an NVFP4 paged cache already holding the
    post-append tokens: q [S, 24, D] -> float32 [S, 24, D]."""
    S = q.shape[0]
    L = pre_len + S
    k = nvfp4.gather_logical_torch(k_cache, k_scales, block_table, L)
    v = nvfp4.gather_logical_torch(v_cache, v_scales, block_table, L)
    return attention_fp32(q, k, v, sm_scale, pre_len)


def draft_split_k(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, length: int,
                  splits: int = 32, block_n: int = 64) -> torch.Tensor:
    """Restates `_partial_kernel` + `_merge_kernel`
    (engine/forward/draft_attention.py:23-79) in FP32.

    q [24, D]; k, v [T, 4, D] float32; chunk = ceil(ceil(length/SPLITS)/64)*64,
    split i covers [i*chunk, min(length, (i+1)*chunk)); partial (acc, m, l)
    with natural-exp online softmax; merge weights exp(m - max), empty
    splits weigh 0.
    """
    scale = DIM ** -0.5
    chunk = math.ceil(math.ceil(length / splits) / block_n) * block_n
    out = torch.zeros(HEADS, DIM)
    for h in range(KV_HEADS):
        qh = q[h * GROUP:(h + 1) * GROUP].float()
        accs, ms, ls = [], [], []
        for i in range(splits):
            start, end = i * chunk, min(length, (i + 1) * chunk)
            if start >= end:
                accs.append(torch.zeros(GROUP, DIM))
                ms.append(torch.full((GROUP,), float("-inf")))
                ls.append(torch.zeros(GROUP))
                continue
            s = qh @ k[start:end, h].float().T * scale
            m = s.max(dim=1).values
            p = torch.exp(s - m[:, None])
            accs.append(p @ v[start:end, h].float())
            ms.append(m)
            ls.append(p.sum(dim=1))
        m = torch.stack(ms)          # [splits, 6]
        top = m.max(dim=0).values
        w = torch.where(m == float("-inf"), torch.zeros_like(m), torch.exp(m - top))
        total = (w * torch.stack(ls)).sum(dim=0)
        acc = (torch.stack(accs) * w[..., None]).sum(dim=0)
        out[h * GROUP:(h + 1) * GROUP] = acc / total[:, None]
    return out


def lse_merge(ms: torch.Tensor, ls: torch.Tensor, os_: torch.Tensor) -> torch.Tensor:
    """Merge of unnormalised partials (log2-domain m): out = sum 2^(m-M) O / sum 2^(m-M) l.
    ms, ls [n, rows]; os_ [n, rows, D]."""
    M = ms.max(dim=0).values
    w = torch.where(ms == float("-inf"), torch.zeros_like(ms), torch.exp2(ms - M))
    return (os_ * w[..., None]).sum(0) / (w * ls).sum(0)[:, None]
