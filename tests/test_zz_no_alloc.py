"""qwz_nvfp4_attend_noalloc — the allocation-free entry point.

Callers that cannot allocate device memory (an engine that owns every
allocation, a fixed memory pool, an FFI that only passes raw pointers) use
this variant: its split-K workspace is a static device array inside the
library instead of caller-supplied buffers.  These tests call it through the
C ABI and check it against qwz_nvfp4_attend, which takes the caller's
workspace, on two consecutive calls (a 7-row verify and then a 1-row decode,
so the second call starts from the array left by the first).  Both entry
points run the same kernels with the same split count, so their outputs must
be bit-identical.  The size limit is checked at its edge: 4,080 records (24
rows x 170 splits, the largest count under 4,096 that 24 rows divide) run and
match, 4,104 (171 splits) are refused.  The file is named so that pytest
collects it last.
"""
from __future__ import annotations


import numpy as np
import pytest
import torch

from oracle import rng
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


def _new_rows(seed, q_len, device):
    def one(s):
        return torch.from_numpy(rng.normal(s, q_len * 1024).astype(np.float32)).view(q_len, 4, 256).half().to(device)
    return one(200 + seed), one(300 + seed)


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
        kn, vn = _new_rows(step, q_len, cuda)
        lens = torch.tensor([start], dtype=torch.int32, device=cuda)
        splits = 20 if q_len == 7 else 37
        out_ref = torch.empty_like(q)
        out_na = torch.empty_like(q)
        _call(lib, "qwz_nvfp4_attend", q, kn, vn, ref_cache, lens, out_ref, splits,
              ops.split_workspace(cuda, q_len, splits))
        _call(lib, "qwz_nvfp4_attend_noalloc", q, kn, vn, na_cache, lens, out_na, splits)
        torch.cuda.synchronize()
        assert torch.equal(out_na, out_ref), f"noalloc call {step + 1} (q_len={q_len}) differs"
        for name in ("k_cache", "v_cache", "k_scales", "v_scales"):
            assert torch.equal(na_cache[name].view(torch.uint8), ref_cache[name].view(torch.uint8)), name
        start += q_len


def test_noalloc_size_limit_at_its_edge(cuda):
    from qwarz_b200 import _lib, ops

    lib = _lib.load()
    pages, pre = 12, 2900
    table = rng.permutation(78, pages)
    c, _, _ = make_cache(78, pre, pages, table)
    ref_cache = to_device(c, cuda)
    na_cache = _clone(ref_cache)
    q = queries(150, 1).to(cuda)
    kn, vn = _new_rows(50, 1, cuda)
    lens = torch.tensor([pre], dtype=torch.int32, device=cuda)
    # 24 x 170 = 4080 records, the most that fit (most splits own no token)
    out_ref = torch.empty_like(q)
    out_na = torch.empty_like(q)
    _call(lib, "qwz_nvfp4_attend", q, kn, vn, ref_cache, lens, out_ref, 170, ops.split_workspace(cuda, 1, 170))
    _call(lib, "qwz_nvfp4_attend_noalloc", q, kn, vn, na_cache, lens, out_na, 170)
    torch.cuda.synchronize()
    assert torch.equal(out_na, out_ref)
    assert _lib.device_error(clear=True) == 0
    # one split more (4104 records), or 8 rows x 22 splits (4224): refused
    # before anything is launched
    p = q.data_ptr()
    for q_len, splits in ((1, 171), (8, 22)):
        rc = lib.qwz_nvfp4_attend_noalloc(*([p] * 10), 1, 1, q_len, splits, 1 / 16, 0, None)
        assert rc == _lib.QWZ_EINVAL
        assert b"static workspace" in lib.qwz_last_error()
