"""GPU parity of the NVFP4 prefill kernel (qwz_nvfp4_prefill) against the
oracle: FP32 softmax attention over the oracle-dequantised pages with the
reference's lower-right causal mask (xqa.py:612-673), through the C ABI."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import rng
from tests.conftest import assert_close_attention
from tests.gpu_helpers import make_cache, queries, to_cpu_torch, to_device

pytestmark = pytest.mark.gpu


def _prefill_case(cuda, seed, pre, S, dtype, spare_pages=1, garbage=True):
    from qwarz_b200 import _lib, ops

    L = pre + S
    pages = (L + 255) // 256 + spare_pages
    table = rng.permutation(seed, pages)
    c, _, _ = make_cache(seed, L, pages, table)
    if garbage:  # bytes past the sequence end are stale (0x7F scales are E4M3 NaN)
        for n in ("k_cache", "v_cache", "k_scales", "v_scales"):
            flat = c[n].reshape(pages * 256, -1)
            phys = np.concatenate([np.arange(table[lp] * 256, table[lp] * 256 + 256) for lp in range(pages)])
            flat[phys[L:]] = 0x7F
    dc = to_device(c, cuda)
    q = queries(seed + 7, S, dtype).to(cuda)
    out = torch.full_like(q, float("nan"))
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    _lib.device_error(clear=True)
    ops.nvfp4_prefill(q, dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"], dc["table"][None],
                      lens, out)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    ref_c = to_cpu_torch(c)
    expect = oatt.nvfp4_attention(q.float().cpu(), ref_c["k_cache"], ref_c["v_cache"], ref_c["k_scales"],
                                  ref_c["v_scales"], ref_c["table"], pre)
    return out.float().cpu().numpy(), expect.numpy()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("pre,S", [(0, 9), (250, 9), (0, 21), (0, 22), (63, 65), (100, 64), (1000, 300)])
def test_prefill_matches_oracle(cuda, dtype, pre, S):
    """Block edges of the kernel: 21 query positions per CTA, 64-token KV
    tiles, 256-token pages crossed; the last tile and page are partly past
    the sequence end and hold NaN-scale garbage."""
    out, expect = _prefill_case(cuda, 300 + pre + S, pre, S, dtype)
    assert_close_attention(out, expect, f"prefill pre={pre} S={S} {dtype}", str(dtype).split(".")[-1])


def test_prefill_long_context(cuda):
    """A 500-token prefill onto 3,000 cached tokens (14 pages, 55 KV tiles)."""
    out, expect = _prefill_case(cuda, 900, 3000, 500, torch.bfloat16, garbage=False)
    assert_close_attention(out, expect, "prefill pre=3000 S=500", "bfloat16")


def test_prefill_single_position(cuda):
    """q_len 1 through the prefill kernel equals decode attention."""
    out, expect = _prefill_case(cuda, 950, 700, 1, torch.float16)
    assert_close_attention(out, expect, "prefill pre=700 S=1", "float16")


def test_prefill_bad_table_entry_is_reported(cuda):
    """A table entry outside the pool: the tile is not loaded, the page-range
    bit is set, and the kernel returns (bounded waits, no hang)."""
    from qwarz_b200 import _lib, ops

    pre, S, pages = 300, 30, 2  # tokens 256.. sit on logical page 1
    table = np.array([1, 7], np.int32)  # page 7 does not exist (pool of 2)
    c, _, _ = make_cache(960, 256, pages, np.array([1, 0], np.int32))
    c["table"] = table
    dc = to_device(c, cuda)
    q = queries(961, S, torch.float16).to(cuda)
    out = torch.zeros_like(q)
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    _lib.device_error(clear=True)
    ops.nvfp4_prefill(q, dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"], dc["table"][None],
                      lens, out)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) & 2  # QWZ_DEVERR_PAGE_RANGE


def test_adapter_prefill_route(cuda):
    """q_len 40 through the public attend(): one append, one prefill launch;
    the cache holds the oracle writer's bytes and the output matches."""
    from oracle import nvfp4
    from qwarz_b200 import attention

    pre, S, pages = 180, 40, 2
    table = np.array([1, 0], np.int32)
    k = rng.normal(970, (pre + S) * 4 * 256).astype(np.float32).reshape(pre + S, 4, 256)
    v = rng.normal(971, (pre + S) * 4 * 256).astype(np.float32).reshape(pre + S, 4, 256)
    k16, v16 = k.astype(np.float16), v.astype(np.float16)
    cpu = {n: np.zeros(s, np.uint8) for n, s in (
        ("k_cache", (pages, 256, 4, 128)), ("v_cache", (pages, 256, 4, 128)),
        ("k_scales", (pages, 256, 4, 16)), ("v_scales", (pages, 256, 4, 16)))}
    nvfp4.append(k16[:pre].astype(np.float32), v16[:pre].astype(np.float32), cpu["k_cache"], cpu["v_cache"],
                 cpu["k_scales"], cpu["v_scales"], table, 0)
    cache = (torch.from_numpy(cpu["k_cache"]).to(cuda), torch.from_numpy(cpu["v_cache"]).to(cuda),
             torch.from_numpy(cpu["k_scales"]).to(cuda).view(torch.float8_e4m3fn),
             torch.from_numpy(cpu["v_scales"]).to(cuda).view(torch.float8_e4m3fn))
    q = queries(972, S, torch.float16).view(1, S, 24, 256)
    out = attention.attend(q.to(cuda), torch.from_numpy(k16[pre:]).view(1, S, 4, 256).to(cuda),
                           torch.from_numpy(v16[pre:]).view(1, S, 4, 256).to(cuda), cache, pre,
                           block_table=torch.from_numpy(table).to(cuda).view(1, -1))
    torch.cuda.synchronize()
    nvfp4.append(k16[pre:].astype(np.float32), v16[pre:].astype(np.float32), cpu["k_cache"], cpu["v_cache"],
                 cpu["k_scales"], cpu["v_scales"], table, pre)
    for name, t in zip(("k_cache", "v_cache", "k_scales", "v_scales"), cache):
        np.testing.assert_array_equal(t.view(torch.uint8).cpu().numpy(), cpu[name], err_msg=name)
    expect = oatt.nvfp4_attention(q[0].float(), *(torch.from_numpy(cpu[n]) for n in
                                  ("k_cache", "v_cache", "k_scales", "v_scales")), torch.from_numpy(table), pre)
    assert_close_attention(out[0].float().cpu().numpy(), expect.numpy(), "attend prefill S=40", "float16")
