"""GPU parity of the draft-model prefill attention (qwz_draft_prefill, the
dense FP16 instantiation of the prefill kernel) against the oracle's FP32
softmax attention with the bottom-right causal mask of
engine/forward/draft.py:33-61 (`draft_attend`), through the C ABI."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import rng
from tests.conftest import assert_close_attention
from tests.gpu_helpers import queries

pytestmark = pytest.mark.gpu


def _kv(seed: int, rows: int) -> torch.Tensor:
    """FP16 [rows, 4, 256] ~ N(0, 1) with four x8 outlier channels per head,
    the draft cache's value distribution in the benchmark configs."""
    x = rng.normal(seed, rows * 4 * 256).astype(np.float32).reshape(rows, 4, 256)
    ch = rng.permutation(seed + 1, 256)[:4]
    x[:, :, ch] *= 8.0
    return torch.from_numpy(x).to(torch.float16)


def _case(cuda, seed, S, T, stride=1024, cap_extra=100):
    """q [1, S, 24, 256]; k, v as [1, T, 4, 256] views (token stride
    `stride` elements) into buffers whose rows past T hold NaN."""
    from qwarz_b200 import _lib
    from qwarz_b200.draft_attention import draft_attend

    cap = T + cap_extra
    bufs = []
    for s in (seed + 1, seed + 2):
        buf = torch.full((cap * stride,), float("nan"), dtype=torch.float16)
        view = buf.as_strided((cap, 4, 256), (stride, 256, 1))
        view[:T] = _kv(s, T)
        bufs.append(buf.to(cuda))
    k = bufs[0].as_strided((1, T, 4, 256), (cap * stride, stride, 256, 1))
    v = bufs[1].as_strided((1, T, 4, 256), (cap * stride, stride, 256, 1))
    q = queries(seed + 3, S, torch.float16).to(cuda)[None]
    _lib.device_error(clear=True)
    out = draft_attend(q, k, v)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    assert out.shape == (1, S, 24, 256) and out.dtype == torch.float16
    expect = oatt.attention_fp32(q[0].float().cpu(), k[0].float().cpu(), v[0].float().cpu(), 256 ** -0.5, T - S)
    return out[0].float().cpu().numpy(), expect.numpy()


@pytest.mark.parametrize("S,T", [(1, 1), (1, 300), (9, 9), (21, 21), (22, 100), (64, 64), (65, 700),
                                 (100, 1000), (300, 300), (257, 2050)])
def test_draft_prefill_matches_oracle(cuda, S, T):
    """The three reference routes in one mask: S == T (square causal),
    S == 1 (every key), S < T (the past plus a causal chunk); block edges at
    21 query rows per CTA and 64-token tiles; rows past T are NaN and must
    read as zeros."""
    out, expect = _case(cuda, 1000 + S + T, S, T)
    assert_close_attention(out, expect, f"draft prefill S={S} T={T}", "float16")


def test_draft_prefill_strided_rows(cuda):
    """A token stride above 1024 elements (1032): the tensor maps take it."""
    out, expect = _case(cuda, 1400, 40, 500, stride=1032)
    assert_close_attention(out, expect, "draft prefill stride 1032", "float16")


def test_draft_prefill_long(cuda):
    """1,024 new rows after 7,168 past rows (128 KV tiles)."""
    out, expect = _case(cuda, 1500, 1024, 8192, cap_extra=0)
    assert_close_attention(out, expect, "draft prefill S=1024 T=8192", "float16")


def test_draft_prefill_rejects_bad_arguments(cuda):
    from qwarz_b200 import ops

    q = torch.zeros(1, 8, 24, 256, dtype=torch.float16, device=cuda)
    kv = torch.zeros(1, 4, 4, 256, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        ops.draft_prefill(q, kv, kv, torch.empty_like(q))  # more query rows than keys
    kb = torch.zeros(1, 16, 4, 256, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        ops.draft_prefill(q, kb, kb, torch.empty_like(q))
