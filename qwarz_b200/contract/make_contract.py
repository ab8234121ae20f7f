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
            # the reference's donor Attention64 row layout for q_len 7, which
            # its ABI test pins (tests/test_attention_kernel_abi.py:51-55); it
            # describes the kernel this library replaces, not one it runs
            "q7_layout": {"BLOCK_M": 8, "BLOCK_H": 2, "BLOCK_ROWS": 16, "programs": 12, "BLOCK_N": 64},
            "q7_layout_scope": "donor Attention64 (replaced); the sm_100a kernels' layout is geometry.b200",
            "b200": {
                "q1": {"kernel": "nvfp4_decode_kernel", "stage_tokens": 256, "stages": 3,
                       "mma": "mma.sync m16n8k16", "mma_m": "16 tokens", "mma_n": "8 (6 GQA heads + 2 pad)",
                       "tokens_per_warp_per_stage": 32},
                "q7": {"kernel": "verify_tc_kernel<VtNvfp4>", "rows": 42, "stage_tokens": 128,
                       "split_bounds": "128-token tiles (a split may start or end mid-page)",
                       "mma": "tcgen05 kind::f16", "qk": "S^T[128 tokens x 48] = K Q^T, K in tensor memory",
                       "pv": "O^T[256 d x 48] += V^T P^T, two M=128 halves of d, V and P in shared memory"},
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
