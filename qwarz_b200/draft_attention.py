"""Draft-model attention for the MTP proposer.

`draft_attend` is the drop-in for engine/forward/draft.py:33-61: q_len new
FP16 rows over the draft's FP16 K/V (bottom-right causal, GQA 6) in one
sm_100a launch that reads K and V in place, for every q_len.  The reference
picks SDPA, an LSE merge of two SDPA calls, or an FP8 repage + sm120 paged
FMHA (draft.py:99-181) by size; the result here is the FP32-softmax value
all three approximate.

One-row decode attention over the FP8 shadow KV follows.

Drop-in for engine/forward/draft_attention.py:82-108 (`DecodeAttention`):
the constructor allocates the split workspace once and `attend` launches the
sm_100a split-K kernel plus the LSE combine, reading the length from a
device tensor, so a 6-step draft roll can be captured in one CUDA graph
(engine/forward/draft.py:440-472).  `shadow_write` replaces the FP8 shadow
update of draft.py:359-366.  Optional per-(256-token page, KV head) FP32
scales generalise the reference's unscaled `_fp8` shadow (scale 1).
"""
from __future__ import annotations

import torch

from . import ops

SPLITS = 37   # 37 splits x 4 KV heads = 148 CTAs, one per SM
KV_HEADS = 4
DIM = 256


def draft_attend(query, key, value):
    """query [1, S, 24, 256] FP16; key, value [1, T, 4, 256] FP16 (T >= S;
    head and dim contiguous, e.g. a [:, :T] view of the preallocated draft
    cache) -> [1, S, 24, 256] FP16, row s attending keys j <= T - S + s."""
    if query.dim() != 4 or query.shape[0] != 1:
        raise ValueError("query must be [1, S, 24, 256]")
    q = query if query.is_contiguous() else query.contiguous()
    out = torch.empty_like(q)
    ops.draft_prefill(q, key, value, out, DIM ** -0.5)
    return out


class DecodeAttention:
    """Reusable workspace; `attend` launches two kernels and allocates nothing."""

    def __init__(self, heads=24, kv_heads=4, dim=256, device="cuda", splits: int = SPLITS):
        if (heads, kv_heads, dim) != (24, 4, 256):
            raise ValueError("draft attention is pinned to 24/4 heads, head_dim 256")
        self.heads = heads
        self.kv_heads = kv_heads
        self.dim = dim
        self.group = heads // kv_heads
        self.splits = int(splits)
        self.part = torch.empty(heads * self.splits * dim, dtype=torch.float32, device=device)
        self.stat = torch.empty(heads * self.splits * 2, dtype=torch.float32, device=device)

    def attend(self, query, k_store, v_store, length, out, k_scale=None, v_scale=None):
        """query [1,1,H,D] FP16; stores [1,T,KV,D] E4M3; length int32 [1]
        (keys [0, length) are attended); out [1,1,H,D] FP16."""
        for t in (k_store, v_store):
            if t.dtype not in (torch.float8_e4m3fn, torch.uint8):
                raise NotImplementedError("the B200 draft kernel reads the FP8 E4M3 shadow store")
        ops.fp8_draft_decode(query, k_store, v_store, length, self.part, self.stat, out,
                             self.splits, k_scale, v_scale)
        return out

    def step(self, query, key, value, k_store, v_store, position, length, out, k_scale=None, v_scale=None):
        """`shadow_write(key, value, ..., position)` then `attend(...)` in two
        launches: the draft kernel writes the new FP16 rows key, value
        [.., 4, 256] at slot position[0] of the stores and attends [0, length)."""
        ops.fp8_draft_step(query, key, value, position, k_store, v_store, length, self.part, self.stat, out,
                           self.splits, k_scale, v_scale)
        return out


def shadow_write(key, value, k8, v8, position, k_scale=None, v_scale=None):
    """FP8 shadow update at slot position[0]: E4M3(clamp(x / scale, +-448))."""
    ops.fp8_shadow_write(key, value, k8, v8, position, k_scale, v_scale)
