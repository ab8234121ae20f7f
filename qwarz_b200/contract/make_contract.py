"""Regenerate qwarz_b200/contract/contract.json from the sources it freezes.

    python -m qwarz_b200.contract.make_contract
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

from . import backend

PKG = Path(__file__).resolve().parents[1]
ROOT = PKG.parent
CONTRACT = Path(__file__).resolve().parent / "contract.json"
FROZEN = [
    "include/qwz_b200.h",
    "qwarz_b200/csrc/attn_split.cu",
    "qwarz_b200/csrc/attn_combine.cu",
    "qwarz_b200/csrc/kv_write.cu",
    "qwarz_b200/csrc/capi.cu",
    "qwarz_b200/csrc/qwz_common.cuh",
    "qwarz_b200/csrc/qwz_kernels.h",
]


def build_contract() -> dict:
    return {
        "abi_reconfirmed": {
            "split_args": list(backend.SPLIT_ARG_NAMES),
            "combine_args": list(backend.COMBINE_ARG_NAMES),
            "graph_patch_split": {
                "3": "block_table",
                "4": "cache_seqlens",
                "11": "split_len int32",
                "12": "num_pages_per_seq int32",
                "13": "num_splits int32",
            },
            "graph_patch_combine": {"4": "num_splits int32"},
            "wrapper": ("qwz_attn_split takes the 15 ABI arguments followed by the two null "
                        "pointer slots global_scratch and profile_scratch, then q_len, "
                        "num_pages, sm_scale, dtype and the stream"),
            "partials": {
                "partial_o": "FP32 [q_len, 24, num_splits, 256], unnormalised O",
                "partial_ml": "FP32 [q_len, 24, num_splits, 2], (m log2-units, l); "
                              "splits without tokens write m = -inf",
            },
        },
        "geometry": {
            # the reference's donor Attention64 row layout for q_len 7 (the
            # kernel this library replaces, tests/test_attention_kernel_abi.py:51-55)
            "q7_layout": {"BLOCK_M": 8, "BLOCK_H": 2, "BLOCK_ROWS": 16, "programs": 12, "BLOCK_N": 64},
            "b200": {
                "q1": {"mma_m": "16 tokens", "mma_n": "8 (6 GQA heads + 2 pad)", "stage_tokens": 64},
                "q7": {"rows": 42, "mma_n": "48 (6 n-tiles)", "stage_tokens": 64,
                       "phase1": "token split", "phase2": "head-dim split"},
            },
        },
        "decode_policy": backend.DECODE_POLICY,
        "sources": [
            {"path": rel, "sha256": hashlib.sha256((ROOT / rel).read_bytes()).hexdigest()}
            for rel in FROZEN
        ],
    }


def main():
    CONTRACT.write_text(json.dumps(build_contract(), indent=2, sort_keys=True) + "\n")
    print(CONTRACT)


if __name__ == "__main__":
    main()
