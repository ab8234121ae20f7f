"""GPU parity of the sm_100a kernels against the oracle and the reference's
golden vectors, through the C ABI (qwarz_b200.ops -> libqwz_b200.so)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import nvfp4, rng
from tests.conftest import assert_close_attention
from tests.golden import cases
from tests.gpu_helpers import make_cache, queries, to_cpu_torch, to_device

pytestmark = pytest.mark.gpu


def _run_attention(dc, q_dev, pre, splits, split_len=0):
    from qwarz_b200 import ops

    dev = q_dev.device
    q_len = q_dev.shape[0]
    lens = torch.tensor([pre], dtype=torch.int32, device=dev)
    po, pml = ops.split_workspace(dev, q_len, splits)
    out = torch.empty_like(q_dev)
    ops.attn_split(q_dev, dc["k_cache"], dc["v_cache"], dc["table"], lens, po, pml,
                   dc["k_scales"], dc["v_scales"], splits, split_len)
    ops.attn_combine(po, pml, out, splits)
    torch.cuda.synchronize()
    return out.float().cpu(), po, pml


# ------------------------------------------------------------------ dequant
@pytest.mark.parametrize("name", sorted(cases.GATHER))
def test_gather_bit_exact_vs_reference(cuda, golden, name):
    from qwarz_b200 import ops

    case = cases.GATHER[name]
    inp = cases.gather_inputs(case)
    ref = golden[f"{name}__out"]
    d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(cuda) for k, v in inp.items()}
    out = torch.zeros(ref.shape, dtype=torch.float16, device=cuda)
    ops.nvfp4_gather(d["packed"], d["scales"], d["table"], d["seq_lens"], out,
                     case["max_tokens"], case["page"])
    got = out.cpu().numpy()
    for b, n in enumerate(case["seq_lens"]):
        np.testing.assert_array_equal(got[b, :n].view(np.uint16), ref[b, :n].view(np.uint16))


# ------------------------------------------------------------------- writer
def _edge_rows(n):
    """Rows exercising the rounding rules: exact E2M1 ties after a unit
    scale, zero blocks, a block whose scale underflows, one that saturates."""
    x = cases.kv_rows(77, n).copy()
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -1.25, -1.75,
                     -2.5, -3.5, -5.0, -0.1], np.float32)
    x[0, 0, 0:16] = ties           # amax 6 -> s = 1 -> scale 1.0 exactly
    x[0, 1, 16:32] = 0.0           # zero block
    x[0, 2, 32:48] = 1e-6          # scale rounds to 0 in E4M3
    x[0, 3, 48:64] = 60000.0       # s > 448 saturates
    x[0, 3, 48] = -60000.0
    return x


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_append_bit_exact(cuda, dtype):
    from qwarz_b200 import ops

    pages, pre, S = 4, 250, 9   # crosses a page boundary
    table = np.array([2, 0, 3, 1], np.int32)
    rows = _edge_rows(S)
    k32 = torch.from_numpy(rows).to(dtype)
    v32 = torch.from_numpy(cases.kv_rows(5, S)).to(dtype)
    ref = {n: np.zeros(s, np.uint8) for n, s in (
        ("k_cache", (pages, 256, 4, 128)), ("v_cache", (pages, 256, 4, 128)),
        ("k_scales", (pages, 256, 4, 16)), ("v_scales", (pages, 256, 4, 16)))}
    nvfp4.append(k32.float().numpy(), v32.float().numpy(), ref["k_cache"], ref["v_cache"],
                 ref["k_scales"], ref["v_scales"], table, pre)
    dc = to_device({**{n: np.zeros_like(a) for n, a in ref.items()}, "table": table}, cuda)
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    ops.nvfp4_append(k32.to(cuda)[None], v32.to(cuda)[None], dc["k_cache"], dc["v_cache"],
                     dc["k_scales"], dc["v_scales"], dc["table"], lens)
    torch.cuda.synchronize()
    for n in ref:
        got = dc[n].view(torch.uint8).cpu().numpy()
        np.testing.assert_array_equal(got, ref[n], err_msg=n)


def test_append_random_bulk_bit_exact(cuda):
    """A whole 4096-token cache written by one bulk append equals the oracle."""
    from qwarz_b200 import ops

    total, pages = 4096, 16
    table = rng.permutation(5, pages)
    ref, k, v = make_cache(9, total, pages, table)
    dc = to_device({**{n: np.zeros_like(ref[n]) for n in ("k_cache", "v_cache", "k_scales", "v_scales")},
                    "table": table}, cuda)
    lens = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.nvfp4_append(torch.from_numpy(k).half().to(cuda), torch.from_numpy(v).half().to(cuda),
                     dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"], dc["table"], lens)
    torch.cuda.synchronize()
    for n in ("k_cache", "v_cache", "k_scales", "v_scales"):
        np.testing.assert_array_equal(dc[n].view(torch.uint8).cpu().numpy(), ref[n], err_msg=n)


def test_fp8_shadow_write_bit_exact(cuda, golden):
    from qwarz_b200 import ops

    cap = 600
    k8 = torch.zeros(cap, 4, 256, dtype=torch.uint8, device=cuda)
    v8 = torch.zeros_like(k8)
    allh = np.arange(65536, dtype=np.uint16).view(np.float16)
    finite = allh[np.isfinite(allh)]
    table = golden["fp8_table"]
    for i, slot in enumerate(range(0, 64)):
        chunk = np.resize(finite[i * 1024:(i + 1) * 1024], 1024).reshape(4, 256)
        kk = torch.from_numpy(chunk.copy()).to(cuda)
        vv = torch.from_numpy((-chunk).copy()).to(cuda)
        pos = torch.tensor([slot], dtype=torch.int32, device=cuda)
        ops.fp8_shadow_write(kk, vv, k8, v8, pos)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(k8[slot].cpu().numpy(), table[chunk.view(np.uint16)])
        np.testing.assert_array_equal(v8[slot].cpu().numpy(), table[(-chunk).view(np.uint16)])
    # with per-(page, head) scales
    ks = torch.tensor(np.array([[0.5, 2.0, 0.01, 3.0]] * 3, np.float32), device=cuda)
    x = torch.from_numpy(cases.kv_rows(3, 1)[0]).half().to(cuda)
    pos = torch.tensor([300], dtype=torch.int32, device=cuda)
    ops.fp8_shadow_write(x, x, k8, v8, pos, ks, ks)
    torch.cuda.synchronize()
    ref = nvfp4.fp8_shadow(x.float().cpu().numpy(), ks[1].cpu().numpy()[:, None])
    np.testing.assert_array_equal(k8[300].cpu().numpy(), ref)


# ---------------------------------------------------------------- attention
@pytest.mark.parametrize("name", sorted(cases.ATTENTION))
def test_attention_vs_reference_golden(cuda, golden, name):
    case = cases.ATTENTION[name]
    inp = cases.attention_inputs(case)
    dc = to_device(inp, cuda)
    q = torch.from_numpy(inp["q"]).to(cuda)
    for splits in (1, 7):
        out, _, _ = _run_attention(dc, q, case["pre"], splits)
        assert_close_attention(out.numpy(), golden[f"{name}__out"], f"{name} splits={splits}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("total", [1, 15, 16, 17, 63, 64, 65, 255, 256, 257, 1000, 4093, 4096])
def test_decode_q1_matches_oracle(cuda, dtype, total):
    pages = 16
    table = rng.permutation(total, pages)
    c, _, _ = make_cache(100 + total, total, pages, table)
    dc = to_device(c, cuda)
    q = queries(total, 1, dtype)
    ref = oatt.nvfp4_attention(q.float(), **{k: v for k, v in to_cpu_torch(c).items() if k != "table"},
                               block_table=torch.from_numpy(table), pre_len=total - 1)
    for splits in (1, 3, 74):
        out, _, _ = _run_attention(dc, q.to(cuda), total - 1, splits)
        assert_close_attention(out.numpy(), ref.numpy(), f"q1 total={total} splits={splits} {dtype}",
                               str(dtype).split(".")[-1])


@pytest.mark.parametrize("q_len", [2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("total", [7, 31, 32, 255, 256, 257, 4093])
def test_verify_matches_oracle(cuda, q_len, total):
    if total < q_len:
        pytest.skip("length shorter than the window")
    pages = 16
    table = rng.permutation(7 * total + q_len, pages)
    c, _, _ = make_cache(200 + total, total, pages, table)
    dc = to_device(c, cuda)
    q = queries(total + q_len, q_len)
    ref = oatt.nvfp4_attention(q.float(), **{k: v for k, v in to_cpu_torch(c).items() if k != "table"},
                               block_table=torch.from_numpy(table), pre_len=total - q_len)
    for splits in (1, 5, 74):
        out, _, _ = _run_attention(dc, q.to(cuda), total - q_len, splits)
        assert_close_attention(out.numpy(), ref.numpy(), f"q{q_len} total={total} splits={splits}")


def test_verify_bf16(cuda):
    total, q_len, pages = 3000, 7, 12
    table = rng.permutation(3, pages)
    c, _, _ = make_cache(31, total, pages, table)
    dc = to_device(c, cuda)
    q = queries(4, q_len, torch.bfloat16)
    ref = oatt.nvfp4_attention(q.float(), **{k: v for k, v in to_cpu_torch(c).items() if k != "table"},
                               block_table=torch.from_numpy(table), pre_len=total - q_len)
    out, _, _ = _run_attention(dc, q.to(cuda), total - q_len, 9)
    assert_close_attention(out.numpy(), ref.numpy(), "q7 bf16", "bfloat16")


def test_fixed_split_len_and_empty_splits(cuda):
    """split_len > 0 (the reference's host-computed chunking) and splits that
    own no token (m = -inf, skipped by the combine)."""
    total, pages = 1300, 8
    table = rng.permutation(8, pages)
    c, _, _ = make_cache(41, total, pages, table)
    dc = to_device(c, cuda)
    q = queries(41, 1)
    ref = oatt.nvfp4_attention(q.float(), **{k: v for k, v in to_cpu_torch(c).items() if k != "table"},
                               block_table=torch.from_numpy(table), pre_len=total - 1)
    out, _, pml = _run_attention(dc, q.to(cuda), total - 1, 12, split_len=256)
    assert_close_attention(out.numpy(), ref.numpy(), "split_len=256")
    ml = pml.view(24, 12, 2).cpu()
    assert torch.isinf(ml[:, 6:, 0]).all() and (ml[:, 6:, 0] < 0).all()   # splits 6.. are empty
    assert torch.isfinite(ml[:, :6, 0]).all()


def test_known_answer_uniform_softmax(cuda):
    """Zero Q and K give a uniform softmax; V[..., 0] = 1,2,3,4 over 4 tokens
    averages to 2.5 (the reference's known answer, tests/test_q38_phases.py:307-320).
    V[..., 1] = 6 pins every block scale to 1.0, so 1..4 are exact E2M1 values."""
    pages = 1
    k = np.zeros((4, 4, 256), np.float32)
    v = np.zeros((4, 4, 256), np.float32)
    v[:, :, 0] = np.array([1, 2, 3, 4], np.float32)[:, None]
    v[:, :, 1] = 6.0
    c = {n: np.zeros(s, np.uint8) for n, s in (
        ("k_cache", (pages, 256, 4, 128)), ("v_cache", (pages, 256, 4, 128)),
        ("k_scales", (pages, 256, 4, 16)), ("v_scales", (pages, 256, 4, 16)))}
    nvfp4.append(k, v, c["k_cache"], c["v_cache"], c["k_scales"], c["v_scales"], np.array([0]), 0)
    c["table"] = np.array([0], np.int32)
    dc = to_device(c, cuda)
    q = torch.zeros(1, 24, 256, dtype=torch.float16, device=cuda)
    out, _, _ = _run_attention(dc, q, 3, 1)
    np.testing.assert_array_equal(out[:, :, 0].numpy(), 2.5)
    np.testing.assert_array_equal(out[:, :, 1].numpy(), 6.0)
    np.testing.assert_array_equal(out[:, :, 2:].numpy(), 0.0)


# ------------------------------------------------- attend (append + attention)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("pre,splits", [(0, 1), (255, 3), (256, 37), (1023, 1), (2900, 1), (2900, 5),
                                        (2900, 37)])
def test_attend_q1_writes_the_row_and_attends_over_it(cuda, dtype, pre, splits):
    """q_len 1 through qwz_nvfp4_attend: the decode kernel writes the new row
    itself.  The pool must hold the oracle writer's bytes and the output must
    match the oracle over it, whether the row's page is one of the owning
    CTA's first three pages (1023/1 is the fourth; 2900/1 the twelfth)."""
    from qwarz_b200 import _lib, ops

    pages = 12
    table = rng.permutation(400 + pre, pages)
    c, _, _ = make_cache(401, pre, pages, table)
    kn = torch.from_numpy(cases.kv_rows(402 + pre, 1)).to(dtype)
    vn = torch.from_numpy(cases.kv_rows(403 + pre, 1)).to(dtype)
    ref = {n: c[n].copy() for n in ("k_cache", "v_cache", "k_scales", "v_scales", "table")}
    nvfp4.append(kn.float().numpy(), vn.float().numpy(), ref["k_cache"], ref["v_cache"],
                 ref["k_scales"], ref["v_scales"], table, pre)
    dc = to_device(c, cuda)
    q = queries(404 + pre, 1, dtype).to(cuda)
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    po, pml = ops.split_workspace(cuda, 1, splits)
    out = torch.empty_like(q)
    _lib.device_error(clear=True)
    ops.nvfp4_attend(q, kn.to(cuda), vn.to(cuda), dc["k_cache"], dc["v_cache"], dc["k_scales"],
                     dc["v_scales"], dc["table"], lens, out, po, pml, splits)
    torch.cuda.synchronize()
    for n in ("k_cache", "v_cache", "k_scales", "v_scales"):
        np.testing.assert_array_equal(dc[n].view(torch.uint8).cpu().numpy(), ref[n], err_msg=n)
    expect = oatt.nvfp4_attention(q.float().cpu(), **{k: v for k, v in to_cpu_torch(ref).items() if k != "table"},
                                  block_table=torch.from_numpy(table), pre_len=pre)
    assert_close_attention(out.float().cpu().numpy(), expect.numpy(),
                           f"attend q1 pre={pre} splits={splits} {dtype}", str(dtype).split(".")[-1])
    assert _lib.device_error(clear=True) == 0


def test_attend_q1_row_beyond_the_table_is_reported(cuda):
    """A full table: the new row has no page.  Nothing is written, the table
    overrun is reported, and the output stays finite."""
    from qwarz_b200 import _lib, ops

    pages, pre = 2, 512
    table = np.array([1, 0], np.int32)
    c, _, _ = make_cache(410, pre, pages, table)
    dc = to_device(c, cuda)
    before = {n: dc[n].clone() for n in ("k_cache", "v_cache", "k_scales", "v_scales")}
    q = queries(411, 1).to(cuda)
    kn = torch.ones(1, 4, 256, dtype=torch.float16, device=cuda)
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    po, pml = ops.split_workspace(cuda, 1, 3)
    out = torch.empty_like(q)
    _lib.device_error(clear=True)
    ops.nvfp4_attend(q, kn, kn, dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"],
                     dc["table"], lens, out, po, pml, 3)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) & 1  # QWZ_DEVERR_TABLE_RANGE
    assert torch.isfinite(out.float()).all()
    for n, t in before.items():
        assert torch.equal(dc[n].view(torch.uint8), t.view(torch.uint8)), n


# -------------------------------------------------------------------- draft
def test_draft_vs_reference_golden(cuda, golden):
    from qwarz_b200.draft_attention import DecodeAttention

    case = cases.DRAFT
    inp = cases.draft_inputs(case)
    q = torch.from_numpy(inp["q"]).view(1, 1, 24, 256).to(cuda)
    k8 = torch.from_numpy(inp["k8"]).to(cuda).view(torch.float8_e4m3fn)[None]
    v8 = torch.from_numpy(inp["v8"]).to(cuda).view(torch.float8_e4m3fn)[None]
    length = torch.tensor([case["length"]], dtype=torch.int32, device=cuda)
    for splits in (16, 32, 5):
        attn = DecodeAttention(24, 4, 256, cuda, splits=splits)
        out = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
        attn.attend(q, k8, v8, length, out)
        torch.cuda.synchronize()
        assert_close_attention(out.float().cpu().numpy(), golden["draft__out"].astype(np.float32),
                               f"draft splits={splits}")


def test_draft_with_page_scales_matches_oracle(cuda):
    from qwarz_b200.draft_attention import DecodeAttention

    T, length = 1100, 1037
    rows_k = cases.kv_rows(61, T)
    rows_v = cases.kv_rows(62, T)
    pages = (T + 255) // 256
    kscale = (np.full((pages, 4), 0.02) * (1 + np.arange(pages * 4).reshape(pages, 4) % 3)).astype(np.float32)
    vscale = (np.full((pages, 4), 0.03) * (1 + np.arange(pages * 4).reshape(pages, 4) % 2)).astype(np.float32)
    k8 = np.zeros((T, 4, 256), np.uint8)
    v8 = np.zeros((T, 4, 256), np.uint8)
    for p in range(pages):
        sl = slice(p * 256, min(T, (p + 1) * 256))
        k8[sl] = nvfp4.fp8_shadow(rows_k[sl], kscale[p][:, None])
        v8[sl] = nvfp4.fp8_shadow(rows_v[sl], vscale[p][:, None])
    kf = torch.from_numpy(nvfp4.e4m3_decode(k8) * np.repeat(kscale, 256, 0)[:T, :, None])
    vf = torch.from_numpy(nvfp4.e4m3_decode(v8) * np.repeat(vscale, 256, 0)[:T, :, None])
    q = queries(63, 1)
    ref = oatt.attention_fp32(q.float(), kf[:length], vf[:length], 1 / 16, length - 1)
    attn = DecodeAttention(24, 4, 256, cuda, splits=16)
    out = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
    attn.attend(q.to(cuda).view(1, 1, 24, 256), torch.from_numpy(k8).to(cuda)[None],
                torch.from_numpy(v8).to(cuda)[None], torch.tensor([length], dtype=torch.int32, device=cuda),
                out, torch.from_numpy(kscale).to(cuda), torch.from_numpy(vscale).to(cuda))
    torch.cuda.synchronize()
    assert_close_attention(out.float().cpu().view(1, 24, 256).numpy(), ref.numpy(), "draft scaled")


@pytest.mark.parametrize("length", [1, 127, 128, 129, 383, 700])
def test_draft_ignores_stale_rows_past_length(cuda, length):
    """Rows at and past `length` hold E4M3 NaN bytes (0x7f): stages are read
    whole, so the kernel must mask their scores and zero their values.  At
    length == capacity the last stage runs past the store and reads the
    copy engine's zero fill."""
    from qwarz_b200.draft_attention import DecodeAttention

    T = 700
    k8 = nvfp4.fp8_shadow(cases.kv_rows(71, T))
    v8 = nvfp4.fp8_shadow(cases.kv_rows(72, T))
    k8[length:] = 0x7F
    v8[length:] = 0x7F
    kf = torch.from_numpy(nvfp4.e4m3_decode(k8[:length]))
    vf = torch.from_numpy(nvfp4.e4m3_decode(v8[:length]))
    q = queries(73, 1)
    ref = oatt.attention_fp32(q.float(), kf, vf, 1 / 16, length - 1)
    kd, vd = torch.from_numpy(k8).to(cuda)[None], torch.from_numpy(v8).to(cuda)[None]
    lens = torch.tensor([length], dtype=torch.int32, device=cuda)
    for splits in (1, 3, 37):
        attn = DecodeAttention(24, 4, 256, cuda, splits=splits)
        out = torch.empty(1, 1, 24, 256, dtype=torch.float16, device=cuda)
        attn.attend(q.to(cuda).view(1, 1, 24, 256), kd, vd, lens, out)
        torch.cuda.synchronize()
        assert_close_attention(out.float().cpu().view(1, 24, 256).numpy(), ref.numpy(),
                               f"draft stale length={length} splits={splits}")


# ------------------------------------------------------------- diagnostics
def test_bad_page_id_sets_device_error_without_fault(cuda):
    """A table entry outside the pool is skipped (zero-filled) and reported
    in the device error word; the context stays usable."""
    from qwarz_b200 import _lib

    total, pages = 600, 3
    table = np.array([0, 1, 2], np.int32)
    c, _, _ = make_cache(51, total, pages, table)
    dc = to_device(c, cuda)
    dc["table"] = torch.tensor([0, 7, 2], dtype=torch.int32, device=cuda)  # 7 is not a page
    _lib.device_error(clear=True)
    out, _, _ = _run_attention(dc, queries(51, 1).to(cuda), total - 1, 3)
    assert _lib.device_error(clear=True) & 2  # QWZ_DEVERR_PAGE_RANGE
    assert np.isfinite(out.numpy()).all()
    # still usable
    dc["table"] = torch.from_numpy(table).to(cuda)
    out2, _, _ = _run_attention(dc, queries(51, 1).to(cuda), total - 1, 3)
    assert np.isfinite(out2.numpy()).all()
    assert _lib.device_error(clear=True) == 0
