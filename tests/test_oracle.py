"""The CPU oracle against the reference's golden vectors and rounding rules
(no GPU)."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4, rng
from tests.golden import cases


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# ------------------------------------------------------- pinned by golden
@pytest.mark.parametrize("name", sorted(cases.GATHER))
def test_gather_matches_reference_kernel_bit_exact(golden, name):
    case = cases.GATHER[name]
    inp = cases.gather_inputs(case)
    assert golden[f"{name}__sha_in"].tobytes().decode() == _sha(*inp.values())
    out = nvfp4.gather(inp["packed"], inp["scales"], inp["table"], inp["seq_lens"],
                       case["max_tokens"], case["page"])
    ref = golden[f"{name}__out"]
    for b, n in enumerate(case["seq_lens"]):
        np.testing.assert_array_equal(out[b, :n].view(np.uint16), ref[b, :n].view(np.uint16))


@pytest.mark.parametrize("name", sorted(cases.ATTENTION))
def test_attention_matches_reference_oracle_route(golden, name):
    case = cases.ATTENTION[name]
    inp = cases.attention_inputs(case)
    assert golden[f"{name}__sha_in"].tobytes().decode() == _sha(*inp.values())
    c = {k: torch.from_numpy(v) for k, v in inp.items()}
    out = oatt.nvfp4_attention(c["q"].float(), c["k_cache"], c["v_cache"], c["k_scales"],
                               c["v_scales"], c["table"], case["pre"])
    np.testing.assert_allclose(out.numpy(), golden[f"{name}__out"], atol=1e-4, rtol=0)


def test_draft_split_k_matches_reference_kernels(golden):
    inp = cases.draft_inputs(cases.DRAFT)
    assert golden["draft__sha_in"].tobytes().decode() == _sha(*inp.values())
    k = torch.from_numpy(nvfp4.e4m3_decode(inp["k8"]))
    v = torch.from_numpy(nvfp4.e4m3_decode(inp["v8"]))
    out = oatt.draft_split_k(torch.from_numpy(inp["q"]).float(), k, v, cases.DRAFT["length"])
    ref = golden["draft__out"][0, 0].astype(np.float32)
    np.testing.assert_allclose(out.numpy(), ref, atol=2e-3, rtol=0)
    # the split-K/LSE merge equals one softmax over all keys
    full = oatt.attention_fp32(torch.from_numpy(inp["q"]).float()[None], k[:650], v[:650], 1 / 16, 649)
    np.testing.assert_allclose(out.numpy(), full[0].numpy(), atol=1e-5, rtol=0)


def test_fp8_shadow_matches_reference_cast_on_every_fp16(golden):
    allh = np.arange(65536, dtype=np.uint16).view(np.float16)
    finite = np.isfinite(allh)
    mine = nvfp4.fp8_shadow(allh.astype(np.float32))
    np.testing.assert_array_equal(mine[finite], golden["fp8_table"][finite])


# --------------------------------------------------------- rounding rules
def test_e4m3_encode_matches_torch_cast():
    """RNE E4M3 of finite floats in range equals torch's float8_e4m3fn cast."""
    x = np.concatenate([
        rng.uniform(1, 200000) * 448.0,
        np.exp(rng.normal(2, 200000) * 4.0) * 0.01,
        np.ldexp(1.0, np.arange(-12, 9)),
        (np.arange(1, 4096) / 512.0),
    ]).astype(np.float32)
    x = x[x < 448.0]
    ours = nvfp4.e4m3_encode_nonneg(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ours, theirs)


def test_e4m3_round_trip_and_saturation():
    b = np.arange(256, dtype=np.uint8)
    finite_pos = b[(b < 0x7F)]
    np.testing.assert_array_equal(nvfp4.e4m3_encode_nonneg(nvfp4.e4m3_decode(finite_pos)), finite_pos)
    assert nvfp4.e4m3_encode_nonneg(np.array([448.0, 464.0, 1e30], np.float32)).tolist() == [0x7E] * 3
    assert nvfp4.e4m3_encode_nonneg(np.array([0.0, 2.0 ** -10, 2.0 ** -10 * 1.0001], np.float32)).tolist() == [0, 0, 1]


def test_e2m1_ties_to_even_and_saturation():
    y = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 7.0, -0.25, -0.3, -5.0, -100.0], np.float32)
    codes = nvfp4.e2m1_encode(y)
    assert codes.tolist() == [0, 2, 2, 4, 4, 6, 6, 7, 7, 0, 9, 14, 15]


def test_quantize_rows_rules():
    x = np.zeros((4, 32), np.float32)
    x[0, :16] = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0]
    x[1, :16] = 1e-6          # scale underflows to 0 -> codes 0
    x[2, :16] = 60000.0       # s > 448 saturates
    packed, scales = nvfp4.quantize_rows(x)
    assert scales[0, 0] == 0x38                       # E4M3(1.0)
    vals = nvfp4.dequant_rows(packed, scales)
    np.testing.assert_array_equal(vals[0, :16], [0, 1, 1, 2, 2, 4, 4, 6, 0, -1, -1, -2, -2, -4, -4, -6])
    assert scales[1, 0] == 0 and not packed[1, :8].any()
    assert scales[2, 0] == 0x7E and (vals[2, :16] == 448.0 * 6.0).all()
    assert scales[3].tolist() == [0, 0] and not packed[3].any()   # zero rows


def test_quantize_error_bound():
    x = cases.kv_rows(5, 64).reshape(-1, 256)
    packed, scales = nvfp4.quantize_rows(x)
    vals = nvfp4.dequant_rows(packed, scales)
    blk = np.abs(x).reshape(-1, 16, 16).max(-1, keepdims=True)
    err = np.abs(vals - x).reshape(-1, 16, 16)
    # half the largest E2M1 step (1 of 2..4 / 2 of 4..6) relative to amax/6,
    # plus the E4M3 scale rounding
    assert (err <= blk * (1.0 / 6.0) * 1.0 * 1.07 + 1e-7).all()


def test_dequant_torch_equals_numpy():
    c = cases.attention_inputs(cases.ATTENTION["attn_q7"])
    a = nvfp4.dequant_rows(c["k_cache"], c["k_scales"])
    b = nvfp4.dequant_rows_torch(torch.from_numpy(c["k_cache"]), torch.from_numpy(c["k_scales"])).numpy()
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    # scales given as float8_e4m3fn (the cache's own dtype) read the same bytes
    f8 = torch.from_numpy(c["k_scales"]).view(torch.float8_e4m3fn)
    b8 = nvfp4.dequant_rows_torch(torch.from_numpy(c["k_cache"]), f8).numpy()
    np.testing.assert_array_equal(a.view(np.uint32), b8.view(np.uint32))


def test_e4m3_decode_torch_equals_numpy_on_every_byte():
    allb = np.arange(256, dtype=np.uint8)
    want = nvfp4.e4m3_decode(allb)
    for t in (torch.from_numpy(allb), torch.from_numpy(allb).view(torch.float8_e4m3fn)):
        got = nvfp4.e4m3_decode_torch(t).numpy()
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    # and torch's own float8 cast agrees on every non-NaN byte
    ref = torch.from_numpy(allb).view(torch.float8_e4m3fn).float().numpy()
    finite = ~np.isnan(want)
    np.testing.assert_array_equal(ref[finite], want[finite])


# ---------------------------------------------------------- attention math
def test_lse_merge_equals_single_softmax():
    q = torch.from_numpy(rng.normal(1, 3 * 24 * 256).astype(np.float32)).view(3, 24, 256)
    k = torch.from_numpy(rng.normal(2, 700 * 4 * 256).astype(np.float32)).view(700, 4, 256)
    v = torch.from_numpy(rng.normal(3, 700 * 4 * 256).astype(np.float32)).view(700, 4, 256)
    full = oatt.attention_fp32(q[:1], k, v, 1 / 16, 699)[0]
    ms, ls, os_ = [], [], []
    for a, b in ((0, 200), (200, 201), (201, 700)):
        s = torch.einsum("hd,thd->ht", q[0], k[a:b].repeat_interleave(6, 1)) / 16 * 1.4426950408889634
        m = s.max(1).values
        p = torch.exp2(s - m[:, None])
        ms.append(m)
        ls.append(p.sum(1))
        os_.append(torch.einsum("ht,thd->hd", p, v[a:b].repeat_interleave(6, 1)))
    ms.append(torch.full((24,), float("-inf")))
    ls.append(torch.zeros(24))
    os_.append(torch.full((24, 256), float("nan")))   # an empty split is never read
    merged = oatt.lse_merge(torch.stack(ms), torch.stack(ls), torch.nan_to_num(torch.stack(os_)))
    np.testing.assert_allclose(merged.numpy(), full.numpy(), atol=1e-5)


def test_lower_right_causal_mask():
    q = torch.ones(3, 24, 256)
    k = torch.zeros(5, 4, 256)
    v = torch.arange(5, dtype=torch.float32)[:, None, None].expand(5, 4, 256).contiguous()
    out = oatt.attention_fp32(q, k, v, 1.0, 2)
    # row s sees keys 0..2+s: uniform mean = (2+s)/2
    assert out[:, 0, 0].tolist() == [1.0, 1.5, 2.0]
