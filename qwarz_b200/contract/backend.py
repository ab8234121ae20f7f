"""Split/combine ABI of libqwz_b200.so in the reference's argument order.

Split (tests/test_attention_kernel_abi.py:16-20): 15 named arguments, then
the two trailing pointer slots the reference's kernel wrapper appends
(global_scratch, profile_scratch).  Arguments 11, 12, 13 are int32 (the
indices a CUDA graph patches per replay in the reference, :25-31); combine
argument 4 (num_splits) is int32.
"""
from __future__ import annotations

import ctypes

from .. import _lib

SPLIT_ARG_NAMES = (
    "q", "k_cache", "v_cache", "block_table", "cache_seqlens", "out",
    "partial_o", "partial_ml", "k_scales", "v_scales", "h32",
    "split_len", "num_pages_per_seq", "num_splits", "sinks",
)
TRAILING_ARG_NAMES = ("global_scratch", "profile_scratch")
INT32_ARG_INDEX = (11, 12, 13)
COMBINE_ARG_NAMES = ("partial_o", "partial_ml", "out", "h32", "num_splits", "sinks")
COMBINE_INT32_ARG_INDEX = (4,)

# Launch policy of the sm_100a kernels (cf. the reference's
# hybrid.DECODE_POLICY for its Triton Attention64 split kernel).
DECODE_POLICY = {
    "q1": {"kernel": "nvfp4_decode_kernel", "warps": 8, "stage_tokens": 256, "stages": 3,
           "copy": "TMA 2-D boxes, 128-byte swizzle", "mma": "mma.sync m16n8k16 tokens x heads(6->8)",
           "ctas_per_sm": 1, "append": "fused when called through qwz_nvfp4_attend"},
    "q2-8": {"kernel": "verify_tc_kernel<VtNvfp4>", "warps": 19,
             "roles": "K TMA, MMA/TMEM owner, V TMA, 16 math (4 per TMEM lane quadrant)",
             "stage_tokens": 128, "stages": {"K": 3, "V": 2}, "copy": "TMA 2-D boxes, 128-byte swizzle",
             "mma": "tcgen05 kind::f16 M=128: S^T = K Q^T (K from TMEM, N=16/32/48), O^T = V^T P^T (FP16 P)",
             "tmem_columns": 512, "ctas_per_sm": 1, "split_bounds": "128-token tiles",
             "append": "fused (the CTAs whose tiles hold the new rows) when called through qwz_nvfp4_attend"},
    "draft": {"kernel": "fp8_draft_kernel", "warps": 8, "stage_tokens": 128, "stages": 3,
              "copy": "TMA 2-D boxes, 128-byte swizzle", "splits": 37,
              "clusters": "2 or 4 CTAs per chunk when chunks x 4 heads leave SMs idle (16 chunks: 2)"},
    "combine": {"kernel": "lse_combine_kernel", "threads": 256, "split_groups": 8},
    "k8v4": {"kernel": "verify_tc_kernel<VtK8v4> (q_len 1..8)", "warps": 19,
             "roles": "K TMA, MMA/TMEM owner, V TMA, 16 math (4 per TMEM lane quadrant)",
             "stage_tokens": 128, "stages": {"K": 2, "V": 2},
             "dequant": "8x8 bit transpose per (token, 32-dim block), fma.rn.f16x2",
             "mma": "tcgen05 kind::f16 M=128 as the NVFP4 verify"},
    "k8v4_combine": {"kernel": "lse_combine_kernel (rotate mode)", "threads": 256, "out": "R^T O per 32 dims"},
}


def pack_split_args(ptrs: dict, ints: dict) -> list[tuple[str, str, int]]:
    """(name, kind, value) for the 15 + 2 split arguments in ABI order; kind
    is "int32" at INT32_ARG_INDEX and "ptr" elsewhere (missing pointers = 0)."""
    packed = []
    for index, name in enumerate(SPLIT_ARG_NAMES + TRAILING_ARG_NAMES):
        if index in INT32_ARG_INDEX:
            value = int(ints[name])
            if not -(1 << 31) <= value < (1 << 31):
                raise ValueError(f"{name} does not fit int32: {value}")
            packed.append((name, "int32", value))
        else:
            packed.append((name, "ptr", int(ptrs.get(name, 0) or 0)))
    return packed


def call_split(packed, q_len: int, num_pages: int, sm_scale: float, dtype: int, stream: int) -> None:
    """Invoke qwz_attn_split with a `pack_split_args` list (stream: cudaStream_t as int)."""
    if [n for n, _, _ in packed] != list(SPLIT_ARG_NAMES + TRAILING_ARG_NAMES):
        raise ValueError("packed arguments are not in ABI order")
    values = [v if k == "int32" else (v or None) for _, k, v in packed]
    lib = _lib.load()
    _lib.check(lib.qwz_attn_split(*values, q_len, num_pages, float(sm_scale), dtype, stream),
               "qwz_attn_split")


def call_k8v4_split(packed, q_len: int, num_pages: int, sm_scale: float, dtype: int, stream: int) -> None:
    """Invoke qwz_k8v4_split (the K8/V4 slot: same 15 + 2 order, h32 given,
    sinks NULL) with a `pack_split_args` list."""
    if [n for n, _, _ in packed] != list(SPLIT_ARG_NAMES + TRAILING_ARG_NAMES):
        raise ValueError("packed arguments are not in ABI order")
    values = [v if k == "int32" else (v or None) for _, k, v in packed]
    lib = _lib.load()
    _lib.check(lib.qwz_k8v4_split(*values, q_len, num_pages, float(sm_scale), dtype, stream), "qwz_k8v4_split")


def call_k8v4_combine(partial_o: int, partial_ml: int, out: int, h32: int, num_splits: int, q_len: int,
                      dtype: int, stream: int) -> None:
    lib = _lib.load()
    _lib.check(lib.qwz_k8v4_combine(partial_o, partial_ml, out, h32, num_splits, None, q_len, dtype, stream),
               "qwz_k8v4_combine")


def call_combine(partial_o: int, partial_ml: int, out: int, num_splits: int, q_len: int,
                 dtype: int, stream: int) -> None:
    lib = _lib.load()
    _lib.check(lib.qwz_attn_combine(partial_o, partial_ml, out, None, num_splits, None, q_len,
                                    dtype, stream), "qwz_attn_combine")


# ------------------------------------------------------------ graph patching
def graph_nodes(graph: int, kind: int) -> list[int]:
    """This library's split (kind 0) or combine (kind 1) kernel nodes of a
    cudaGraph_t (an int handle, e.g. torch's CUDAGraph(keep_graph=True)
    .raw_cuda_graph()), in the graph's node order."""
    lib = _lib.load()
    count = ctypes.c_int32(0)
    _lib.check(lib.qwz_graph_kernel_nodes(graph, kind, None, 0, ctypes.byref(count)), "qwz_graph_kernel_nodes")
    nodes = (ctypes.c_void_p * max(count.value, 1))()
    _lib.check(lib.qwz_graph_kernel_nodes(graph, kind, nodes, count.value, ctypes.byref(count)),
               "qwz_graph_kernel_nodes")
    return [int(nodes[i]) for i in range(count.value)]


def patch_split(graph: int, graph_exec: int | None, node: int, packed) -> None:
    """Patch the graph-patch indices of one captured split node (3, 4, 11,
    12, 13: block_table, cache_seqlens, split_len, num_pages_per_seq,
    num_splits) from a `pack_split_args` list."""
    values = {name: value for name, _, value in packed}
    lib = _lib.load()
    _lib.check(lib.qwz_graph_patch_split(graph, graph_exec, node, values["block_table"], values["cache_seqlens"],
                                         values["split_len"], values["num_pages_per_seq"], values["num_splits"]),
               "qwz_graph_patch_split")


def patch_combine(graph: int, graph_exec: int | None, node: int, num_splits: int) -> None:
    """Patch combine argument 4 (num_splits) of one captured combine node."""
    lib = _lib.load()
    _lib.check(lib.qwz_graph_patch_combine(graph, graph_exec, node, num_splits), "qwz_graph_patch_combine")
