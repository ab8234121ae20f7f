"""ctypes binding of libqwz_b200.so (the C ABI of include/qwz_b200.h).

Follows the reference's own precedent for native code (a shared library
loaded through ctypes, engine/forward/gdn.py:21-39).  There is no fallback:
if the library is missing or fails to load, every operator raises.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int32, c_int64, c_void_p, c_char_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqwz_b200.so"

QWZ_OK = 0
QWZ_EINVAL = -1
QWZ_ELAUNCH = -2
DTYPE_F16 = 0
DTYPE_BF16 = 1
NODE_SPLIT = 0
NODE_COMBINE = 1

_i32p = POINTER(c_int32)
_f32p = POINTER(c_float)

# name -> argtypes (restype is int unless listed in _RESTYPE)
SIGNATURES = {
    "qwz_version": [],
    "qwz_last_error": [],
    "qwz_device_error": [_i32p, c_int32],
    "qwz_nvfp4_append": [c_void_p] * 8 + [c_int32] * 7 + [c_void_p],
    "qwz_nvfp4_append_shard": [c_void_p] * 8 + [c_int32] * 5 + [c_void_p],
    "qwz_attn_split": [c_void_p] * 11 + [c_int32] * 3 + [c_void_p] * 3 + [c_int32, c_int32, c_float, c_int32, c_void_p],
    "qwz_attn_combine": [c_void_p] * 4 + [c_int32, c_void_p, c_int32, c_int32, c_void_p],
    "qwz_nvfp4_attend": [c_void_p] * 12 + [c_int32] * 4 + [c_float, c_int32, c_void_p],
    "qwz_nvfp4_attend_noalloc": [c_void_p] * 10 + [c_int32] * 4 + [c_float, c_int32, c_void_p],
    "qwz_nvfp4_prefill": [c_void_p] * 8 + [c_int32] * 3 + [c_float, c_int32, c_void_p],
    "qwz_draft_prefill": [c_void_p] * 4 + [c_int32] * 2 + [c_int64] * 2 + [c_float, c_void_p],
    "qwz_attn_shard_partial": [c_void_p] * 10 + [c_int32] * 6 + [c_float, c_int32, c_void_p],
    "qwz_lse_combine_gathered": [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p],
    "qwz_fp8_draft_decode": [c_void_p] * 9 + [c_int32, c_int32, c_void_p],
    "qwz_fp8_draft_step": [c_void_p] * 12 + [c_int32, c_int32, c_void_p],
    "qwz_fp8_shadow_write": [c_void_p] * 7 + [c_int32, c_int32, c_void_p],
    "qwz_nvfp4_gather": [c_void_p] * 5 + [c_int32] * 6 + [c_void_p],
    "qwz_peer_buffer_bytes": [c_int32, c_int32],
    "qwz_peer_alloc": [c_int64, POINTER(c_void_p), c_void_p],
    "qwz_peer_open": [c_void_p, POINTER(c_void_p)],
    "qwz_peer_close": [c_void_p],
    "qwz_peer_free": [c_void_p],
    "qwz_attn_shard_split": [c_void_p] * 11 + [c_int32] * 6 + [c_float, c_int32, c_void_p],
    "qwz_shard_exchange_combine": [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int64, c_void_p,
                                   c_int32, c_int32, c_void_p, c_int64, c_int32, c_void_p],
    "qwz_graph_kernel_nodes": [c_void_p, c_int32, c_void_p, c_int32, _i32p],
    "qwz_graph_patch_split": [c_void_p] * 5 + [c_int32] * 3,
    "qwz_graph_patch_combine": [c_void_p] * 3 + [c_int32],
    "qwz_k8v4_append": [c_void_p] * 8 + [c_int32] * 4 + [c_void_p],
    "qwz_k8v4_split": [c_void_p] * 11 + [c_int32] * 3 + [c_void_p] * 3 + [c_int32, c_int32, c_float, c_int32, c_void_p],
    "qwz_k8v4_combine": [c_void_p] * 4 + [c_int32, c_void_p, c_int32, c_int32, c_void_p],
    "qwz_k8v4_gather": [c_void_p] * 3 + [c_int32] * 4 + [c_void_p, c_void_p],
    "qwz_shard_exchange_combine_emulated": [c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p,
                                            c_int64, c_void_p, c_void_p, c_int32, c_int64, c_int32,
                                            c_void_p],
}
_RESTYPE = {"qwz_version": c_char_p, "qwz_last_error": c_char_p, "qwz_peer_buffer_bytes": c_int64}

_LIB = None


class QwzError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


class QwzArgumentError(QwzError, ValueError):
    """The library rejected an argument (QWZ_EINVAL); nothing was launched."""


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with typed entry points."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = Path(path) if path is not None else LIB_PATH
    if not path.exists():
        raise QwzError(
            f"{path} is missing: build it with `python -m qwarz_b200.build` "
            "(the CUDA path has no fallback)")
    lib = ctypes.CDLL(str(path))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPE.get(name, c_int32)
    _LIB = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc == QWZ_OK:
        return
    msg = load().qwz_last_error().decode(errors="replace")
    if rc == QWZ_EINVAL:
        raise QwzArgumentError(f"{what}: {msg}")
    raise QwzError(f"{what}: {msg} (status {rc})")


def device_error(clear: bool = True) -> int:
    """Device error word (QWZ_DEVERR_* bits); synchronises the device."""
    out = c_int32(0)
    check(load().qwz_device_error(ctypes.byref(out), int(clear)), "qwz_device_error")
    return out.value
