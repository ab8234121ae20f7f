"""pytest configuration: the `gpu` marker and shared helpers.

CPU tests (`-m "not gpu"`) cover the oracle against the golden vectors, the
host logic and the C ABI surface.  GPU tests (`-m gpu`) are the parity tests
proper: they call the sm_100a kernels through the C ABI and compare with the
oracle.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device with the library loaded (built first if needed)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwarz_b200 import build, _lib

    build.build()
    _lib.load()
    torch.cuda.init()
    return torch.device("cuda", 0)


def err_stats(out, ref):
    """max-abs, normwise max-rel (max|err| / max|ref|) and rel-L2 of two arrays."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(out - ref)
    max_abs = float(err.max()) if err.size else 0.0
    scale = float(np.abs(ref).max()) if ref.size else 1.0
    max_rel = max_abs / max(scale, 1e-30)
    rel_l2 = float(np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30))
    return max_abs, max_rel, rel_l2


# Attention tolerance of the north star: within max-abs 2e-3 and max-rel
# 1e-2 of an FP32 softmax.  max-rel is normwise (max|err| / max|ref|).  The
# kernels return FP16/BF16, which cannot hold the FP32 reference closer than
# half a unit in the last place (3.9e-3 at |O| = 10 in FP16), so each element
# may also differ by one ulp of the output dtype at |ref|.  rel-L2 is held to
# the reference's own numeric gate, 3e-3 (relative L2 vs an FP32 oracle).
ATOL = 2e-3
RTOL = 1e-2
REL_L2 = 3e-3


def ulp(ref, dtype: str):
    a = np.abs(np.asarray(ref, dtype=np.float64))
    if dtype == "float16":
        return np.spacing(a.astype(np.float16)).astype(np.float64)
    if dtype == "bfloat16":
        e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
        return np.ldexp(1.0, (e - 7).astype(np.int64))
    return np.zeros_like(a)


def assert_close_attention(out, ref, what="", dtype: str = "float16"):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    max_abs, max_rel, rel_l2 = err_stats(out, ref)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    excess = np.abs(out - ref) - (ATOL + ulp(ref, dtype))
    worst = float(excess.max()) if excess.size else 0.0
    assert worst <= 0 and max_rel <= RTOL and rel_l2 <= REL_L2, (
        f"{what}: max_abs={max_abs:.3e} (beyond 2e-3+1ulp by {max(worst, 0):.3e}) "
        f"max_rel={max_rel:.3e} rel_l2={rel_l2:.3e}")
    return max_abs, max_rel, rel_l2
