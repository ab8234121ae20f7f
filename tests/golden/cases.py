"""Seeded inputs of the golden cases (shared by make_golden.py and the tests).

Every input is a pure function of the case dict through oracle.rng, so the
committed golden.npz only stores outputs and SHA-256 digests of the inputs.
"""
from __future__ import annotations

import numpy as np

from oracle import nvfp4, rng

GATHER = {
    # generic geometry of the reference kernel: small head_dim, 2 pages of 256
    "gather_d64": dict(seed=11, pages=2, page=256, heads=4, dim=64,
                       table=[[1, 0]], seq_lens=[300], max_tokens=300),
    # production head_dim, small pages, two sequences with ragged lengths
    "gather_d256": dict(seed=12, pages=5, page=16, heads=4, dim=256,
                        table=[[3, 0, 4, 1, 2], [2, 4, 1, 0, 3]], seq_lens=[70, 33],
                        max_tokens=70),
}

ATTENTION = {
    # MTP verify width 7, causal inside the window, partial last page
    "attn_q7": dict(seed=21, q_len=7, pre=500, pages=3, table=[2, 0, 1]),
    # single-token decode on the CPU-runnable BASELINE geometry (4096 tokens,
    # 16 pages in a seed-permuted table, 4 outlier channels x8)
    "attn_q1_4k": dict(seed=22, q_len=1, pre=4095, pages=16, table="perm"),
    # ragged: length 1 (only the appended token), q_len 1
    "attn_q1_len1": dict(seed=23, q_len=1, pre=0, pages=1, table=[0]),
}

DRAFT = dict(seed=31, capacity=700, length=650)


def _scale_bytes(seed: int, n: int) -> np.ndarray:
    """Random E4M3 bytes without the NaN patterns (0x7F, 0xFF)."""
    b = rng.bytes_(seed, n)
    return np.where((b & 0x7F) == 0x7F, b ^ 0x01, b).astype(np.uint8)


def gather_inputs(case: dict) -> dict:
    s, P, page, H, D = case["seed"], case["pages"], case["page"], case["heads"], case["dim"]
    packed = rng.bytes_(s, P * page * H * D // 2).reshape(P, page, H, D // 2)
    scales = _scale_bytes(s + 1, P * page * H * D // 16).reshape(P, page, H, D // 16)
    return {
        "packed": packed,
        "scales": scales,
        "table": np.array(case["table"], dtype=np.int32),
        "seq_lens": np.array(case["seq_lens"], dtype=np.int32),
    }


def kv_rows(seed: int, n: int, outliers: int = 4) -> np.ndarray:
    """float32 [n, 4, 256] ~N(0,1) with `outliers` seed-chosen channels x8."""
    x = rng.normal(seed, n * 4 * 256).astype(np.float32).reshape(n, 4, 256)
    if outliers:
        ch = rng.permutation(seed + 7, 256)[:outliers]
        x[..., ch] *= 8.0
    return x


def attention_inputs(case: dict) -> dict:
    s, P, S, pre = case["seed"], case["pages"], case["q_len"], case["pre"]
    table = rng.permutation(s + 3, P) if case["table"] == "perm" else np.array(case["table"], np.int32)
    total = pre + S
    q = rng.normal(s, S * 24 * 256).astype(np.float16).reshape(S, 24, 256)
    k_cache = np.zeros((P, 256, 4, 128), np.uint8)
    v_cache = np.zeros((P, 256, 4, 128), np.uint8)
    k_scales = np.zeros((P, 256, 4, 16), np.uint8)
    v_scales = np.zeros((P, 256, 4, 16), np.uint8)
    k = kv_rows(s + 1, total).astype(np.float16).astype(np.float32)
    v = kv_rows(s + 2, total).astype(np.float16).astype(np.float32)
    nvfp4.append(k, v, k_cache, v_cache, k_scales, v_scales, table, 0)
    return {"q": q, "k_cache": k_cache, "v_cache": v_cache, "k_scales": k_scales,
            "v_scales": v_scales, "table": table.astype(np.int32)}


def draft_inputs(case: dict) -> dict:
    s, T = case["seed"], case["capacity"]
    q = rng.normal(s, 24 * 256).astype(np.float16).reshape(24, 256)
    k = (kv_rows(s + 1, T) * 0.5).astype(np.float16)
    v = kv_rows(s + 2, T).astype(np.float16)
    return {"q": q, "k8": nvfp4.fp8_shadow(k), "v8": nvfp4.fp8_shadow(v)}
