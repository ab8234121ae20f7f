"""Builders shared by the GPU parity tests: seeded NVFP4 caches written by the
oracle quantiser (CPU), copied to the device."""
from __future__ import annotations

import numpy as np
import torch

from oracle import nvfp4, rng
from tests.golden import cases


def make_cache(seed: int, total: int, pages: int, table, outliers: int = 4, dtype=np.float16):
    """Oracle-written NVFP4 cache of `total` tokens; returns numpy dict and
    the float32 rows it quantised."""
    table = np.asarray(table, dtype=np.int32)
    k = cases.kv_rows(seed + 1, total, outliers).astype(dtype).astype(np.float32)
    v = cases.kv_rows(seed + 2, total, outliers).astype(dtype).astype(np.float32)
    c = {name: np.zeros(shape, np.uint8) for name, shape in (
        ("k_cache", (pages, 256, 4, 128)), ("v_cache", (pages, 256, 4, 128)),
        ("k_scales", (pages, 256, 4, 16)), ("v_scales", (pages, 256, 4, 16)))}
    nvfp4.append(k, v, c["k_cache"], c["v_cache"], c["k_scales"], c["v_scales"], table, 0)
    c["table"] = table
    return c, k, v


def to_device(c: dict, device):
    d = {name: torch.from_numpy(np.ascontiguousarray(c[name])).to(device)
         for name in ("k_cache", "v_cache", "k_scales", "v_scales")}
    d["k_scales"] = d["k_scales"].view(torch.float8_e4m3fn)
    d["v_scales"] = d["v_scales"].view(torch.float8_e4m3fn)
    d["table"] = torch.from_numpy(np.ascontiguousarray(c["table"])).to(device)
    return d


def to_cpu_torch(c: dict):
    return {name: torch.from_numpy(np.ascontiguousarray(c[name]))
            for name in ("k_cache", "v_cache", "k_scales", "v_scales", "table")}


def queries(seed: int, q_len: int, dtype=torch.float16):
    q = rng.normal(seed, q_len * 24 * 256).astype(np.float32).reshape(q_len, 24, 256)
    return torch.from_numpy(q).to(dtype)
