"""GPU tests of the fused draft step (qwz_fp8_draft_step): the FP8 shadow
write of engine/forward/draft.py:359-366 done inside the draft decode
kernel.  It must equal the two-kernel sequence fp8_shadow_write + the draft
decode bit for bit (same stores, same output), and the oracle within the
attention tolerance."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4
from tests.golden import cases
from tests.conftest import assert_close_attention
from tests.gpu_helpers import queries

pytestmark = pytest.mark.gpu


def _stores(cuda, T, seed, scaled):
    k8 = nvfp4.fp8_shadow(cases.kv_rows(seed, T))
    v8 = nvfp4.fp8_shadow(cases.kv_rows(seed + 1, T))
    pages = (T + 255) // 256
    ks = vs = None
    if scaled:
        ks = torch.from_numpy((0.02 * (1 + np.arange(pages * 4) % 3)).astype(np.float32).reshape(pages, 4)).to(cuda)
        vs = torch.from_numpy((0.03 * (1 + np.arange(pages * 4) % 2)).astype(np.float32).reshape(pages, 4)).to(cuda)
    return (torch.from_numpy(k8).to(cuda).view(torch.float8_e4m3fn)[None],
            torch.from_numpy(v8).to(cuda).view(torch.float8_e4m3fn)[None], ks, vs)


@pytest.mark.parametrize("base", [0, 126, 250, 300, 4095])
@pytest.mark.parametrize("scaled", [False, True])
def test_fused_step_equals_write_then_attend(cuda, base, scaled):
    """A six-step roll (slots base .. base+5, length = slot + 1) across stage
    (128) and page (256) boundaries: stores and outputs are bit-identical to
    fp8_shadow_write followed by the draft decode."""
    from qwarz_b200.draft_attention import DecodeAttention, shadow_write

    T = 4200
    k_a, v_a, ks, vs = _stores(cuda, T, 500 + base, scaled)
    k_b, v_b = k_a.clone(), v_a.clone()
    g = torch.Generator(device="cpu").manual_seed(base)
    attn = DecodeAttention(24, 4, 256, cuda, splits=37)
    for i in range(6):
        slot = base + i
        q = queries(900 + slot, 1).to(cuda).view(1, 1, 24, 256)
        kn = (torch.randn(4, 256, generator=g) * 3).half().to(cuda)
        vn = (torch.randn(4, 256, generator=g) * 3).half().to(cuda)
        pos = torch.tensor([slot], dtype=torch.int32, device=cuda)
        length = torch.tensor([slot + 1], dtype=torch.int32, device=cuda)
        out_a = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
        out_b = torch.empty_like(out_a)
        shadow_write(kn, vn, k_a[0], v_a[0], pos, ks, vs)
        attn.attend(q, k_a, v_a, length, out_a, ks, vs)
        attn.step(q, kn, vn, k_b, v_b, pos, length, out_b, ks, vs)
        torch.cuda.synchronize()
        assert torch.equal(k_a.view(torch.uint8), k_b.view(torch.uint8)), f"K store differs at step {i}"
        assert torch.equal(v_a.view(torch.uint8), v_b.view(torch.uint8)), f"V store differs at step {i}"
        assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16)), f"output differs at step {i}"


def test_fused_step_matches_oracle(cuda):
    """One step at slot 1,036 (length 1,037) against FP32 attention over the
    oracle's FP8 shadow of every row, the new one included."""
    from qwarz_b200.draft_attention import DecodeAttention

    T, slot = 1100, 1036
    rows_k = cases.kv_rows(81, T).astype(np.float16).astype(np.float32)  # the new row arrives as FP16
    rows_v = cases.kv_rows(82, T).astype(np.float16).astype(np.float32)
    k8 = nvfp4.fp8_shadow(rows_k)
    v8 = nvfp4.fp8_shadow(rows_v)
    k8[slot] = 0x7F  # stale bytes where the new row goes
    v8[slot] = 0x7F
    kn = rows_k[slot].astype(np.float16)
    vn = rows_v[slot].astype(np.float16)
    ref_k = nvfp4.fp8_shadow(rows_k)
    ref_v = nvfp4.fp8_shadow(rows_v)
    kf = torch.from_numpy(nvfp4.e4m3_decode(ref_k[:slot + 1]))
    vf = torch.from_numpy(nvfp4.e4m3_decode(ref_v[:slot + 1]))
    q = queries(83, 1)
    ref = oatt.attention_fp32(q.float(), kf, vf, 1 / 16, slot)
    kd = torch.from_numpy(k8).to(cuda).view(torch.float8_e4m3fn)[None]
    vd = torch.from_numpy(v8).to(cuda).view(torch.float8_e4m3fn)[None]
    attn = DecodeAttention(24, 4, 256, cuda, splits=16)
    out = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
    attn.step(q.to(cuda).view(1, 1, 24, 256), torch.from_numpy(kn).to(cuda), torch.from_numpy(vn).to(cuda),
              kd, vd, torch.tensor([slot], dtype=torch.int32, device=cuda),
              torch.tensor([slot + 1], dtype=torch.int32, device=cuda), out)
    torch.cuda.synchronize()
    assert np.array_equal(kd[0, slot].view(torch.uint8).cpu().numpy(), ref_k[slot])
    assert_close_attention(out.float().cpu().view(1, 24, 256).numpy(), ref.numpy(), "fused draft step")


def test_fused_step_slot_past_length_is_written_not_attended(cuda):
    from qwarz_b200 import _lib
    from qwarz_b200.draft_attention import DecodeAttention

    T, length, slot = 900, 500, 610
    k_a, v_a, _, _ = _stores(cuda, T, 700, False)
    k_b, v_b = k_a.clone(), v_a.clone()
    kn = torch.randn(4, 256, device=cuda).half()
    vn = torch.randn(4, 256, device=cuda).half()
    q = queries(701, 1).to(cuda).view(1, 1, 24, 256)
    lens = torch.tensor([length], dtype=torch.int32, device=cuda)
    attn = DecodeAttention(24, 4, 256, cuda, splits=37)
    out_a = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
    out_b = torch.empty_like(out_a)
    attn.attend(q, k_a, v_a, lens, out_a)
    _lib.device_error(clear=True)
    attn.step(q, kn, vn, k_b, v_b, torch.tensor([slot], dtype=torch.int32, device=cuda), lens, out_b)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16))
    expect = nvfp4.fp8_shadow(kn.float().cpu().numpy())
    assert np.array_equal(k_b[0, slot].view(torch.uint8).cpu().numpy(), expect)
    k_b[0, slot] = k_a[0, slot]
    assert torch.equal(k_a.view(torch.uint8), k_b.view(torch.uint8))


def test_fused_step_slot_out_of_range_is_reported(cuda):
    from qwarz_b200 import _lib
    from qwarz_b200.draft_attention import DecodeAttention

    T = 300
    k8, v8, _, _ = _stores(cuda, T, 710, False)
    before = k8.clone()
    attn = DecodeAttention(24, 4, 256, cuda, splits=4)
    out = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
    kn = torch.zeros(4, 256, device=cuda).half()
    _lib.device_error(clear=True)
    attn.step(queries(711, 1).to(cuda).view(1, 1, 24, 256), kn, kn, k8, v8,
              torch.tensor([T], dtype=torch.int32, device=cuda), torch.tensor([T], dtype=torch.int32, device=cuda),
              out)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) & 4  # kErrSlotRange
    assert torch.equal(before.view(torch.uint8), k8.view(torch.uint8))
