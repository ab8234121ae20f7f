"""qwz_nvfp4_attend_noalloc — the allocation-free entry point.

Callers that cannot allocate device memory (an engine that owns every
allocation, a fixed memory pool, an FFI that only passes raw pointers) use
this variant: its split-K workspace is a static device array inside the
library instead of caller-supplied buffers.  These tests call it through the
C ABI and check it against qwz_nvfp4_attend, which takes the caller's
workspace, on two consecutive calls (a 7-row verify and then a 1-row decode,
so the second call starts from the array left by the first).  The file is
named so that pytest collects it last.
"""
from __future__ import annotations


import numpy as np
import pytest
import torch

from oracle import rng
from tests.conftest import assert_close_attention
from tests.gpu_helpers import make_cache, queries, to_device

pytestmark = pytest.mark.gpu


def _clone(dc):
    return {k: v.clone() for k, v in dc.items()}


def _call(lib, fn_name, q, k, v, dc, lens, out, splits, workspace=None):
    stream = torch.cuda.current_stream().cuda_stream
    P = dc["k_cache"].shape[0]
    q_len = q.shape[0]
    common = [q.data_ptr(), k.data_ptr(), v.data_ptr(), dc["k_cache"].data_ptr(),
              dc["v_cache"].data_ptr(), dc["k_scales"].data_ptr(), dc["v_scales"].data_ptr(),
              dc["table"].data_ptr(), lens.data_ptr(), out.data_ptr()]
    if workspace is None:
        rc = getattr(lib, fn_name)(*common, dc["table"].numel(), P, q_len, splits, 1 / 16, 0, stream)
    else:
        po, pml = workspace
        rc = getattr(lib, fn_name)(*common, po.data_ptr(), pml.data_ptr(), dc["table"].numel(), P,
                                   q_len, splits, 1 / 16, 0, stream)
    assert rc == 0, lib.qwz_last_error().decode()


def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda):
    from qwarz_b200 import _lib, ops

    lib = _lib.load()
    pages, pre = 12, 2900
    table = rng.permutation(77, pages)
    c, _, _ = make_cache(77, pre, pages, table)
    ref_cache = to_device(c, cuda)
    na_cache = _clone(ref_cache)
    start = pre
    for step, q_len in enumerate((7, 1)):
        q = queries(100 + step, q_len).to(cuda)
        kn = torch.from_numpy(rng.normal(200 + step, q_len * 1024).astype(np.float32)).view(q_len, 4, 256).half().to(cuda)
        vn = torch.from_numpy(rng.normal(300 + step, q_len * 1024).astype(np.float32)).view(q_len, 4, 256).half().to(cuda)
        lens = torch.tensor([start], dtype=torch.int32, device=cuda)
        splits = 20 if q_len == 7 else 37
        out_ref = torch.empty_like(q)
        out_na = torch.empty_like(q)
        _call(lib, "qwz_nvfp4_attend", q, kn, vn, ref_cache, lens, out_ref, splits,
              ops.split_workspace(cuda, q_len, splits))
        _call(lib, "qwz_nvfp4_attend_noalloc", q, kn, vn, na_cache, lens, out_na, splits)
        torch.cuda.synchronize()
        assert_close_attention(out_na.float().cpu().numpy(), out_ref.float().cpu().numpy(),
                               f"noalloc call {step + 1} (q_len={q_len})")
        for name in ("k_cache", "v_cache", "k_scales", "v_scales"):
            assert torch.equal(na_cache[name].view(torch.uint8), ref_cache[name].view(torch.uint8)), name
        start += q_len


def test_noalloc_refuses_requests_beyond_the_static_workspace(cuda):
    from qwarz_b200 import _lib

    lib = _lib.load()
    dummy = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
    p = dummy.data_ptr()
    # 8 rows x 24 heads x 22 splits = 4224 records > 4096
    rc = lib.qwz_nvfp4_attend_noalloc(*([p] * 10), 1, 1, 8, 22, 1 / 16, 0, None)
    assert rc == _lib.QWZ_EINVAL
    assert b"static workspace" in lib.qwz_last_error()
