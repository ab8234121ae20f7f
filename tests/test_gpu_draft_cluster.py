"""GPU tests of the cluster form of the FP8 draft decode: with too few chunks
to give every SM a CTA (BASELINE's 16 chunks are 64 CTAs on 148 SMs), each
chunk is streamed by a cluster of 2 or 4 CTAs whose (M, l, O) records are
merged through distributed shared memory.  The chunk count, the workspace
and the combine are those of the reference's split-K draft
(engine/forward/draft_attention.py:23-79); the results must match the FP32
oracle, repeat bit for bit, and the fused shadow write must land the same
bytes and output as write-then-attend whichever rank of the cluster streams
the slot's stage."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4
from tests.conftest import assert_close_attention
from tests.golden import cases
from tests.gpu_helpers import queries

pytestmark = pytest.mark.gpu


def _cluster_size(cuda, splits: int) -> int:
    """The launcher's choice: SMs // (chunks x 4 KV heads), 3 rounded down to 2, at most 4."""
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    cl = max(1, min(4, sms // (splits * 4)))
    return 2 if cl == 3 else cl


@pytest.mark.parametrize("splits", [2, 8, 12, 16, 18, 37])
@pytest.mark.parametrize("length", [5, 300, 2100, 9000])
def test_cluster_draft_matches_oracle_and_repeats(cuda, splits, length):
    """Chunk counts that select clusters of 4 (2, 8), 2 (12, 16, 18) and no
    cluster (37); short lengths leave some ranks without a stage."""
    from qwarz_b200.draft_attention import DecodeAttention

    T = 9100
    k8 = nvfp4.fp8_shadow(cases.kv_rows(301, T))
    v8 = nvfp4.fp8_shadow(cases.kv_rows(302, T))
    kf = torch.from_numpy(nvfp4.e4m3_decode(k8[:length]))
    vf = torch.from_numpy(nvfp4.e4m3_decode(v8[:length]))
    q = queries(303 + splits, 1)
    ref = oatt.attention_fp32(q.float(), kf, vf, 1 / 16, length - 1)
    kd, vd = torch.from_numpy(k8).to(cuda)[None], torch.from_numpy(v8).to(cuda)[None]
    lens = torch.tensor([length], dtype=torch.int32, device=cuda)
    attn = DecodeAttention(24, 4, 256, cuda, splits=splits)
    outs = []
    for _ in range(2):
        out = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
        attn.attend(q.to(cuda).view(1, 1, 24, 256), kd, vd, lens, out)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16)), "repeated call differs"
    assert_close_attention(outs[0].float().cpu().view(1, 24, 256).numpy(), ref.numpy(),
                           f"draft splits={splits} (cluster {_cluster_size(cuda, splits)}) length={length}")
    from qwarz_b200 import _lib
    assert _lib.device_error(clear=True) == 0


@pytest.mark.parametrize("splits", [4, 16])
def test_cluster_draft_with_page_scales_matches_oracle(cuda, splits):
    """Per-(page, KV head) FP32 scales: K scales S, V scales P, in every rank."""
    from qwarz_b200.draft_attention import DecodeAttention

    T, length = 3000, 2900
    k8 = nvfp4.fp8_shadow(cases.kv_rows(311, T))
    v8 = nvfp4.fp8_shadow(cases.kv_rows(312, T))
    pages = (T + 255) // 256
    ks = (0.05 * (1 + np.arange(pages * 4) % 5)).astype(np.float32).reshape(pages, 4)
    vs = (0.07 * (1 + np.arange(pages * 4) % 3)).astype(np.float32).reshape(pages, 4)
    tok_page = np.arange(length) // 256
    kf = torch.from_numpy(nvfp4.e4m3_decode(k8[:length]) * ks[tok_page][:, :, None])
    vf = torch.from_numpy(nvfp4.e4m3_decode(v8[:length]) * vs[tok_page][:, :, None])
    q = queries(313, 1)
    ref = oatt.attention_fp32(q.float(), kf, vf, 1 / 16, length - 1)
    attn = DecodeAttention(24, 4, 256, cuda, splits=splits)
    out = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
    attn.attend(q.to(cuda).view(1, 1, 24, 256), torch.from_numpy(k8).to(cuda)[None],
                torch.from_numpy(v8).to(cuda)[None], torch.tensor([length], dtype=torch.int32, device=cuda), out,
                torch.from_numpy(ks).to(cuda), torch.from_numpy(vs).to(cuda))
    torch.cuda.synchronize()
    assert_close_attention(out.float().cpu().view(1, 24, 256).numpy(), ref.numpy(), f"scaled draft splits={splits}")


@pytest.mark.parametrize("splits", [4, 16])
@pytest.mark.parametrize("base", [3, 1150, 4090])
def test_cluster_fused_step_equals_write_then_attend(cuda, splits, base):
    """Six fused steps (slots base .. base+5, length = slot + 1): the new row
    sits in the last stage, which the last rank of the last chunk streams;
    stores and outputs are bit-identical to fp8_shadow_write + attend."""
    from qwarz_b200.draft_attention import DecodeAttention, shadow_write

    T = 4200
    k_a = torch.from_numpy(nvfp4.fp8_shadow(cases.kv_rows(321 + base, T))).to(cuda).view(torch.float8_e4m3fn)[None]
    v_a = torch.from_numpy(nvfp4.fp8_shadow(cases.kv_rows(322 + base, T))).to(cuda).view(torch.float8_e4m3fn)[None]
    k_b, v_b = k_a.clone(), v_a.clone()
    g = torch.Generator(device="cpu").manual_seed(base + splits)
    attn = DecodeAttention(24, 4, 256, cuda, splits=splits)
    for i in range(6):
        slot = base + i
        q = queries(330 + slot, 1).to(cuda).view(1, 1, 24, 256)
        kn = (torch.randn(4, 256, generator=g) * 3).half().to(cuda)
        vn = (torch.randn(4, 256, generator=g) * 3).half().to(cuda)
        pos = torch.tensor([slot], dtype=torch.int32, device=cuda)
        length = torch.tensor([slot + 1], dtype=torch.int32, device=cuda)
        out_a = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
        out_b = torch.empty_like(out_a)
        shadow_write(kn, vn, k_a[0], v_a[0], pos)
        attn.attend(q, k_a, v_a, length, out_a)
        attn.step(q, kn, vn, k_b, v_b, pos, length, out_b)
        torch.cuda.synchronize()
        assert torch.equal(k_a.view(torch.uint8), k_b.view(torch.uint8)), f"K store differs at step {i}"
        assert torch.equal(v_a.view(torch.uint8), v_b.view(torch.uint8)), f"V store differs at step {i}"
        assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16)), f"output differs at step {i}"


def test_cluster_fused_step_slot_past_length_written_once(cuda):
    """A slot past the attended length: only rank 0 of chunk 0 writes it."""
    from qwarz_b200 import _lib
    from qwarz_b200.draft_attention import DecodeAttention

    T, length, slot = 900, 500, 610
    k_a = torch.from_numpy(nvfp4.fp8_shadow(cases.kv_rows(341, T))).to(cuda).view(torch.float8_e4m3fn)[None]
    v_a = torch.from_numpy(nvfp4.fp8_shadow(cases.kv_rows(342, T))).to(cuda).view(torch.float8_e4m3fn)[None]
    k_b, v_b = k_a.clone(), v_a.clone()
    kn = torch.randn(4, 256, device=cuda).half()
    vn = torch.randn(4, 256, device=cuda).half()
    q = queries(343, 1).to(cuda).view(1, 1, 24, 256)
    lens = torch.tensor([length], dtype=torch.int32, device=cuda)
    attn = DecodeAttention(24, 4, 256, cuda, splits=16)
    out_a = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
    out_b = torch.empty_like(out_a)
    attn.attend(q, k_a, v_a, lens, out_a)
    _lib.device_error(clear=True)
    attn.step(q, kn, vn, k_b, v_b, torch.tensor([slot], dtype=torch.int32, device=cuda), lens, out_b)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16))
    assert np.array_equal(k_b[0, slot].view(torch.uint8).cpu().numpy(), nvfp4.fp8_shadow(kn.float().cpu().numpy()))
    assert np.array_equal(v_b[0, slot].view(torch.uint8).cpu().numpy(), nvfp4.fp8_shadow(vn.float().cpu().numpy()))
    k_b[0, slot] = k_a[0, slot]
    v_b[0, slot] = v_a[0, slot]
    assert torch.equal(k_a.view(torch.uint8), k_b.view(torch.uint8))
    assert torch.equal(v_a.view(torch.uint8), v_b.view(torch.uint8))
