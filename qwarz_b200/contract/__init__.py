"""The attention-kernel ABI contract of the reference, re-created for this package.

The reference freezes its split/combine kernel ABI in
``results/20260911-attention-kernel/{backend.py,contract.json}`` and asserts
it in tests/test_attention_kernel_abi.py and
tests/test_attention_kernel_contract.py; those fixtures are gitignored and
absent from the reference tree.  `backend` and `contract.json` here restate
them for libqwz_b200.so (the same 15 + 2 argument order, the int32 graph-patch
indices, the combine ABI), so the reference's assertions run against this
package (tests/test_contract_abi.py).
"""
from .backend import (COMBINE_ARG_NAMES, COMBINE_INT32_ARG_INDEX, DECODE_POLICY,
                      INT32_ARG_INDEX, SPLIT_ARG_NAMES, TRAILING_ARG_NAMES, call_combine,
                      call_split, pack_split_args)

__all__ = ["SPLIT_ARG_NAMES", "TRAILING_ARG_NAMES", "INT32_ARG_INDEX", "COMBINE_ARG_NAMES",
           "COMBINE_INT32_ARG_INDEX", "DECODE_POLICY", "pack_split_args", "call_split",
           "call_combine"]
