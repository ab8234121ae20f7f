"""qwarz_b200 — B200-native (sm_100a) NVFP4-KV paged decode / MTP-verify attention.

A drop-in for the attention hot path of the Qwarz engine:
  attention         `attend`, `empty_cache`, `NVFP4AttentionAdapter`, ... —
                    the engine-facing boundary (engine/forward/attention.py,
                    src/qwasar_runtime/xqa.py)
  draft_attention   `DecodeAttention` over the FP8 shadow KV
                    (engine/forward/draft_attention.py)
  sharded           sequence-page sharding over the GPUs of one node (new)
  ops               torch wrappers of the C ABI (include/qwz_b200.h)
  contract          the split/combine ABI fixtures the reference tests assert
The kernels live in libqwz_b200.so, built from csrc/ by `python -m qwarz_b200.build`.
"""
from . import _lib
from ._lib import QwzArgumentError, QwzError

__all__ = ["QwzError", "QwzArgumentError", "load_library"]


def load_library():
    """Load libqwz_b200.so (raises QwzError if it has not been built)."""
    return _lib.load()
