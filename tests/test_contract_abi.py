"""The reference's attention-kernel ABI/contract assertions
(tests/test_attention_kernel_abi.py, tests/test_attention_kernel_contract.py)
run against this package's re-created fixtures (qwarz_b200/contract)."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

from qwarz_b200.contract import INT32_ARG_INDEX, SPLIT_ARG_NAMES, pack_split_args
from qwarz_b200.contract import backend, make_contract

ROOT = Path(__file__).resolve().parents[1]
CONTRACT = ROOT / "qwarz_b200" / "contract" / "contract.json"


def test_split_abi_has_fifteen_args_and_graph_patches():
    abi = json.loads(CONTRACT.read_text())["abi_reconfirmed"]
    assert len(abi["split_args"]) == 15
    assert abi["split_args"] == [
        "q", "k_cache", "v_cache", "block_table", "cache_seqlens", "out",
        "partial_o", "partial_ml", "k_scales", "v_scales", "h32",
        "split_len", "num_pages_per_seq", "num_splits", "sinks",
    ]
    assert abi["combine_args"] == [
        "partial_o", "partial_ml", "out", "h32", "num_splits", "sinks",
    ]
    assert abi["graph_patch_split"] == {
        "3": "block_table",
        "4": "cache_seqlens",
        "11": "split_len int32",
        "12": "num_pages_per_seq int32",
        "13": "num_splits int32",
    }
    assert abi["graph_patch_combine"] == {"4": "num_splits int32"}
    assert "two null pointer slots" in abi["wrapper"]


def test_pack_split_args_uses_int32_at_graph_patch_indices():
    packed = pack_split_args(
        {name: 0x1000 + i for i, name in enumerate(SPLIT_ARG_NAMES)},
        {"split_len": 1024, "num_pages_per_seq": 1008, "num_splits": 28},
    )
    assert [name for name, _, _ in packed][:15] == list(SPLIT_ARG_NAMES)
    assert len(packed) == 17
    for index in INT32_ARG_INDEX:
        assert packed[index][1] == "int32"
    assert packed[11] == ("split_len", "int32", 1024)
    assert packed[12] == ("num_pages_per_seq", "int32", 1008)
    assert packed[13] == ("num_splits", "int32", 28)
    assert packed[15][0] == "global_scratch"
    assert packed[16][0] == "profile_scratch"


def test_q7_row_layout_matches_donor_attention64():
    geometry = json.loads(CONTRACT.read_text())["geometry"]["q7_layout"]
    assert geometry == {
        "BLOCK_M": 8, "BLOCK_H": 2, "BLOCK_ROWS": 16, "programs": 12, "BLOCK_N": 64,
    }


def test_contract_matches_sources_and_policy():
    """Like the reference contract test: policy and every frozen source hash."""
    contract = json.loads(CONTRACT.read_text())
    assert contract["decode_policy"] == json.loads(json.dumps(backend.DECODE_POLICY))
    for source in contract["sources"]:
        path = ROOT / source["path"]
        assert path.is_file(), path
        assert hashlib.sha256(path.read_bytes()).hexdigest() == source["sha256"], (
            f"{source['path']} changed: rerun python -m qwarz_b200.contract.make_contract")
    abi = contract["abi_reconfirmed"]
    assert abi["split_args"][3:5] == ["block_table", "cache_seqlens"]
    assert abi["split_args"][11:14] == ["split_len", "num_pages_per_seq", "num_splits"]
    assert abi["graph_patch_split"]["13"] == "num_splits int32"
    assert abi["graph_patch_combine"]["4"] == "num_splits int32"
    assert contract == json.loads(json.dumps(make_contract.build_contract()))


def test_c_header_declares_split_in_abi_order():
    header = (ROOT / "include" / "qwz_b200.h").read_text()
    start = header.index("int qwz_attn_split(")
    decl = header[start:header.index(");", start)]
    names = [part.strip().split()[-1].lstrip("*") for part in decl[len("int qwz_attn_split("):].split(",")]
    assert names[:15] == list(SPLIT_ARG_NAMES)
    assert names[15:17] == ["global_scratch", "profile_scratch"]
    start = header.index("int qwz_attn_combine(")
    decl = header[start:header.index(");", start)]
    names = [part.strip().split()[-1].lstrip("*") for part in decl[len("int qwz_attn_combine("):].split(",")]
    assert names[:6] == list(backend.COMBINE_ARG_NAMES)
