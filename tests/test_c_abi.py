"""The C-ABI library loads and exports what include/qwz_b200.h declares; the
host-side argument checks reject bad calls without launching (no GPU)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from qwarz_b200 import _lib, build

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qwz_b200.h"


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(qwz_\w+)\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "qwz_attn_split" in names and "qwz_attn_combine" in names
    assert len(names) >= 12


def test_library_exports_every_declared_symbol(lib):
    for name in declared():
        assert hasattr(lib, name), name
    assert set(declared()) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_signature_arity_matches_header():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, argtypes in _lib.SIGNATURES.items():
        m = re.search(rf"{name}\((.*?)\);", text, flags=re.S)
        assert m, name
        body = m.group(1).strip()
        arity = 0 if body in ("", "void") else body.count(",") + 1
        assert arity == len(argtypes), name


def test_version(lib):
    assert b"sm_100a" in lib.qwz_version()


def _rc_and_msg(lib, rc):
    return rc, lib.qwz_last_error().decode()


def test_split_rejects_null_and_k8v4_features(lib):
    rc, msg = _rc_and_msg(lib, lib.qwz_attn_split(*([None] * 11), 0, 1, 1, *([None] * 3), 1, 1,
                                                  0.0625, 0, None))
    assert rc == _lib.QWZ_EINVAL and "q must" in msg
    buf = ctypes.create_string_buffer(4096 + 64)
    addr = (ctypes.addressof(buf) + 63) // 64 * 64
    ptrs = [addr] * 11
    ptrs[10] = addr  # h32 set
    rc, msg = _rc_and_msg(lib, lib.qwz_attn_split(*ptrs, 0, 1, 1, None, None, None, 1, 1, 0.0625, 0, None))
    assert rc == _lib.QWZ_EINVAL and "h32" in msg


@pytest.mark.parametrize("q_len,splits,split_len,scale,dtype,needle", [
    (0, 4, 0, 0.0625, 0, "q_len"),
    (9, 4, 0, 0.0625, 0, "q_len"),
    (1, 0, 0, 0.0625, 0, "num_splits"),
    (1, 4, 100, 0.0625, 0, "split_len"),
    (1, 4, 0, -1.0, 0, "sm_scale"),
    (1, 4, 0, 0.0625, 7, "dtype"),
])
def test_split_argument_checks(lib, q_len, splits, split_len, scale, dtype, needle):
    buf = ctypes.create_string_buffer(4096 + 64)
    addr = (ctypes.addressof(buf) + 63) // 64 * 64
    ptrs = [addr] * 10 + [None]
    rc, msg = _rc_and_msg(lib, lib.qwz_attn_split(*ptrs, split_len, 4, splits, None, None, None,
                                                  q_len, 16, scale, dtype, None))
    assert rc == _lib.QWZ_EINVAL and needle in msg


def test_misaligned_cache_rejected(lib):
    buf = ctypes.create_string_buffer(4096 + 64)
    addr = (ctypes.addressof(buf) + 63) // 64 * 64
    ptrs = [addr] * 10 + [None]
    ptrs[1] = addr + 4
    rc, msg = _rc_and_msg(lib, lib.qwz_attn_split(*ptrs, 0, 4, 4, None, None, None, 1, 16, 0.0625, 0, None))
    assert rc == _lib.QWZ_EINVAL and "aligned" in msg


def test_writer_geometry_is_pinned(lib):
    buf = ctypes.create_string_buffer(4096 + 64)
    addr = (ctypes.addressof(buf) + 63) // 64 * 64
    rc, msg = _rc_and_msg(lib, lib.qwz_nvfp4_append(*([addr] * 8), 4, 1, 4, 64, 256, 4, 0, None))
    assert rc == _lib.QWZ_EINVAL and "page 256" in msg


def test_python_ops_refuse_cpu_tensors():
    import torch
    from qwarz_b200 import ops

    q = torch.zeros(1, 24, 256, dtype=torch.float16)
    cache = (torch.zeros(1, 256, 4, 128, dtype=torch.uint8),) * 2 + (torch.zeros(1, 256, 4, 16, dtype=torch.uint8),) * 2
    with pytest.raises(ValueError, match="CUDA"):
        ops.attn_split(q, cache[0], cache[1], torch.zeros(1, 1, dtype=torch.int32),
                       torch.zeros(1, dtype=torch.int32), torch.zeros(1), torch.zeros(1),
                       cache[2], cache[3], 1)


def test_peer_buffer_size_and_exchange_argument_checks(lib):
    rows = 24
    assert lib.qwz_peer_buffer_bytes(1, 1) == 2 * rows * 258 * 8
    assert lib.qwz_peer_buffer_bytes(8, 2) == 2 * 8 * 2 * rows * 258 * 8
    assert lib.qwz_peer_buffer_bytes(0, 1) == 0 and lib.qwz_peer_buffer_bytes(9, 1) == 0
    assert lib.qwz_peer_buffer_bytes(2, 9) == 0
    buf = ctypes.create_string_buffer(4096 + 64)
    addr = (ctypes.addressof(buf) + 63) // 64 * 64
    peers = (ctypes.c_uint64 * 2)(addr, addr)
    pv = ctypes.cast(peers, ctypes.c_void_p)
    nb = lib.qwz_peer_buffer_bytes(2, 1)
    for world, rank, q_len, splits, p, nbytes, timeout, needle in [
            (9, 0, 1, 4, pv, nb, 0, "world"), (2, 2, 1, 4, pv, nb, 0, "rank"), (2, 0, 0, 4, pv, nb, 0, "q_len"),
            (2, 0, 1, 0, pv, nb, 0, "num_splits"), (2, 0, 1, 4, None, nb, 0, "peers"),
            # buffers sized for another (world, q_len): refused before any store
            (2, 0, 2, 4, pv, nb, 0, "buffer_bytes"), (4, 0, 1, 4, pv, nb, 0, "buffer_bytes"),
            (2, 0, 1, 4, pv, nb + 8, 0, "buffer_bytes"),
            (2, 0, 1, 4, pv, nb, -1, "timeout_ns"), (2, 0, 1, 4, pv, nb, 10**10 + 1, "timeout_ns")]:
        rc, msg = _rc_and_msg(lib, lib.qwz_shard_exchange_combine(addr, addr, splits, q_len, p, nbytes, addr, rank,
                                                                  world, addr, timeout, 0, None))
        assert rc == _lib.QWZ_EINVAL and needle in msg, (needle, msg)
    bad = (ctypes.c_uint64 * 2)(addr + 8, addr)
    rc, msg = _rc_and_msg(lib, lib.qwz_shard_exchange_combine(addr, addr, 4, 1, ctypes.cast(bad, ctypes.c_void_p),
                                                              nb, addr, 0, 2, addr, 0, 0, None))
    assert rc == _lib.QWZ_EINVAL and "16-byte aligned" in msg
    rc, msg = _rc_and_msg(lib, lib.qwz_shard_exchange_combine_emulated(
        addr, addr, 4, 4, 1, pv, nb + 1, addr, addr, 2, 0, 0, None))
    assert rc == _lib.QWZ_EINVAL and "buffer_bytes" in msg
    rc, msg = _rc_and_msg(lib, lib.qwz_attn_shard_split(*([addr] * 11), 4, 1, 100, 256, 1, 4, 0.0625, 0, None))
    assert rc == _lib.QWZ_EINVAL and "tok_begin" in msg


def test_prefill_draft_prefill_and_draft_step_argument_checks(lib):
    buf = ctypes.create_string_buffer(4096 + 64)
    a = (ctypes.addressof(buf) + 63) // 64 * 64
    # qwz_nvfp4_prefill(q, kc, vc, ks, vs, table, lens, out, table_width, pages, q_len, sm_scale, dtype, stream)
    for tw, q_len, scale, needle in [(0, 4, 0.0625, "table_width"), (1, 0, 0.0625, "q_len"),
                                     (1, 4, 0.0, "sm_scale")]:
        rc, msg = _rc_and_msg(lib, lib.qwz_nvfp4_prefill(*([a] * 8), tw, 1, q_len, scale, 0, None))
        assert rc == _lib.QWZ_EINVAL and needle in msg, (needle, msg)
    # qwz_draft_prefill(q, k, v, out, q_len, kv_len, k_stride, v_stride, sm_scale, stream)
    for args, needle in [((a, None, a, a, 4, 8, 1024, 1024, 0.0625), "k and v"),
                         ((a, a, a, a, 9, 8, 1024, 1024, 0.0625), "q_len <= kv_len"),
                         ((a, a, a, a, 4, 8, 1000, 1024, 0.0625), "token strides"),
                         ((a, a, a, a, 4, 8, 1024, 1028, 0.0625), "token strides"),
                         ((a, a, a, a, 4, 8, 1024, 1024, -1.0), "sm_scale")]:
        rc, msg = _rc_and_msg(lib, lib.qwz_draft_prefill(*args, None))
        assert rc == _lib.QWZ_EINVAL and needle in msg, (needle, msg)
    # qwz_fp8_draft_step(q, k_new, v_new, position, k8, v8, ks, vs, length, part, stat, out, splits, cap, stream)
    rc, msg = _rc_and_msg(lib, lib.qwz_fp8_draft_step(a, None, a, a, a, a, None, None, a, a, a, a, 4, 256, None))
    assert rc == _lib.QWZ_EINVAL and "k_new" in msg
    rc, msg = _rc_and_msg(lib, lib.qwz_fp8_draft_step(a, a, a, None, a, a, None, None, a, a, a, a, 4, 256, None))
    assert rc == _lib.QWZ_EINVAL and "position" in msg
    rc, msg = _rc_and_msg(lib, lib.qwz_fp8_draft_step(a, a, a, a, a, a, None, None, a, a, a, a, 0, 256, None))
    assert rc == _lib.QWZ_EINVAL and "splits" in msg


def test_draft_prefill_ops_refuse_cpu_and_non_fp16():
    import torch
    from qwarz_b200 import ops

    q = torch.zeros(1, 8, 24, 256, dtype=torch.float16)
    kv = torch.zeros(1, 16, 4, 256, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.draft_prefill(q, kv, kv, torch.empty_like(q))


def test_graph_patch_argument_checks(lib):
    count = ctypes.c_int32(-1)
    rc, msg = _rc_and_msg(lib, lib.qwz_graph_kernel_nodes(None, 0, None, 0, ctypes.byref(count)))
    assert rc == _lib.QWZ_EINVAL and "graph" in msg
    buf = ctypes.create_string_buffer(64)
    rc, msg = _rc_and_msg(lib, lib.qwz_graph_kernel_nodes(ctypes.addressof(buf), 7, None, 0, ctypes.byref(count)))
    assert rc == _lib.QWZ_EINVAL and "kind" in msg
    rc, msg = _rc_and_msg(lib, lib.qwz_graph_kernel_nodes(ctypes.addressof(buf), 0, None, 4, ctypes.byref(count)))
    assert rc == _lib.QWZ_EINVAL and "nodes" in msg
    p = ctypes.addressof(buf)
    for args, needle in (((None, None, None, p, p, 0, 4, 8), "node"),
                         ((None, None, p, None, p, 0, 4, 8), "block_table"),
                         ((None, None, p, p, p, 0, 0, 8), "num_pages_per_seq"),
                         ((None, None, p, p, p, 0, 4, 0), "num_splits"),
                         ((None, None, p, p, p, 100, 4, 8), "split_len")):
        rc, msg = _rc_and_msg(lib, lib.qwz_graph_patch_split(*args))
        assert rc == _lib.QWZ_EINVAL and needle in msg, (needle, msg)
    for args, needle in (((None, None, None, 4), "node"), ((None, None, p, 0), "num_splits")):
        rc, msg = _rc_and_msg(lib, lib.qwz_graph_patch_combine(*args))
        assert rc == _lib.QWZ_EINVAL and needle in msg, (needle, msg)
