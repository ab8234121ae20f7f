"""Drop-in attention boundary over the NVFP4 one-level KV cache.

Mirrors the reference operator the engine calls:
  * `attend(q, k, v, cache, cache_len)`, `empty_cache`, `bind_table_pages`,
    `cache_seqlens`, `release_attention_plans`
    (engine/forward/attention.py:144-250);
  * `NVFP4AttentionAdapter` with the same validation, append ownership,
    decline rule, per-(layer, q_len) CUDA graphs, route counters and
    diagnostics (src/qwasar_runtime/xqa.py:240-906);
  * `install`, prepending the adapter to a dispatcher list and restoring it
    (xqa.py:909-920).
The decode/verify route (q_len <= 8) is one append + one split-K launch +
one combine of the sm_100a kernels in libqwz_b200.so; there is no CPU
fallback.  q_len > 8 (prefill) runs the NVFP4 prefill kernel after one append.
"""
from __future__ import annotations

import dataclasses
import weakref
from collections import Counter
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any

import torch

from . import ops

DONOR_PAGE_SIZE = 256
XQA_MAX_QUERY = 8
HEADS = 24
KV_HEADS = 4
HEAD_DIM = 256
PAGE = 256


def _capturing() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


@dataclass
class AttnArgs:
    """The ExLlamaV3 `AttnArgs` fields the reference adapter reads
    (xqa.py:307-354, attention.py:226-248)."""

    bsz: int
    q_len: int
    num_q_heads: int
    dim: int
    kv_len: int
    num_kv_heads: int
    q: torch.Tensor
    k: torch.Tensor | None
    v: torch.Tensor | None
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    causal: bool
    sm_scale: float
    cu_seqlens: Any = None
    max_seqlen: Any = None
    window_size: Any = None
    softcap: float = 0.0
    block_table: torch.Tensor | None = None
    cache_seqlens: torch.Tensor | None = None
    k_scales: torch.Tensor | None = None
    v_scales: torch.Tensor | None = None
    non_causal_spans: Any = None
    sinks: Any = None

    def is_varlen(self) -> bool:
        return self.cu_seqlens is not None

    def _replace(self, **kwargs) -> "AttnArgs":
        return dataclasses.replace(self, **kwargs)


@dataclass
class _LayerState:
    outputs: dict = field(default_factory=dict)
    workspaces: dict = field(default_factory=dict)
    graphs: dict = field(default_factory=dict)
    graph_calls: Counter = field(default_factory=Counter)


@dataclass
class _Graph:
    """Per-(layer, q_len) CUDA graph owning append + split + combine.

    q/k/v/lengths/table stage through static tensors copied before each
    replay (the generator rebuilds the table every cycle, xqa.py:169-173);
    the cache tensors are bound through weak references and checked on every
    replay, so a rebuilt cache drops and recaptures the graph (xqa.py:175-197).
    """

    graph: Any
    static_q: torch.Tensor
    static_k: torch.Tensor
    static_v: torch.Tensor
    static_seqlens: torch.Tensor
    static_table: torch.Tensor
    output: torch.Tensor | None
    bound_caches: tuple | None = None
    failed: bool = False

    def matches(self, args) -> bool:
        if self.failed or self.bound_caches is None:
            return False
        return (self.bound_caches[0]() is args.k_cache and self.bound_caches[1]() is args.v_cache
                and self.bound_caches[2]() is args.k_scales and self.bound_caches[3]() is args.v_scales
                and tuple(self.static_table.shape) == tuple(args.block_table.shape))


class NVFP4AttentionAdapter:
    """One process-local attention candidate with explicit append ownership."""

    XQA_GRAPH_WARMUPS = 3
    QUERY_DTYPES = (torch.float16,)

    def __init__(self, mode: str = "nvfp4-b200", flashinfer_module: Any = None,
                 prefill: str = "sdpa", decode_graphs: bool = True,
                 query_dtypes: tuple = (torch.float16,)):
        if mode not in ("nvfp4-b200", "nvfp4-xqa", "nvfp4-triton"):
            raise ValueError(f"unsupported mode: {mode}")
        if prefill not in ("sdpa", "prims"):
            raise ValueError(f"unsupported prefill route: {prefill}")
        self.mode = mode
        self.prefill = prefill
        self.decode_graphs = decode_graphs
        self.query_dtypes = tuple(query_dtypes)
        self.routes: Counter[str] = Counter()
        self.query_rows: Counter[str] = Counter()
        self.layer_states: dict = {}
        self.max_observed_query = 0
        self.append_calls = 0
        self._host_cache_len = None

    # ------------------------------------------------------------ contract
    def _validate_nvfp4(self, args) -> int:
        """Same checks and messages as xqa.py:307-354 (FP16 queries by
        default; BF16 when the adapter was built with it in query_dtypes)."""
        if args.bsz != 1:
            raise ValueError("Qwasar NVFP4 adapter is deliberately restricted to batch size 1")
        if args.is_varlen() or args.non_causal_spans is not None:
            raise ValueError("Qwasar NVFP4 adapter does not support varlen or non-causal spans")
        if not args.causal:
            raise ValueError("Qwasar NVFP4 adapter requires causal attention")
        if args.window_size not in (None, -1):
            raise ValueError("Qwasar full-attention layers must not use a sliding window")
        if args.softcap not in (None, 0, 0.0) or args.sinks is not None:
            raise ValueError("Qwasar adapter does not support softcap or attention sinks")
        if args.q.dtype not in self.query_dtypes or not args.q.is_contiguous():
            raise ValueError("XQA experiment requires contiguous FP16 queries")
        if args.dim != 256 or args.num_q_heads != 24 or args.num_kv_heads != 4:
            raise ValueError("XQA experiment is pinned to Q24/KV4/D256")
        if args.k_cache.dtype != torch.uint8 or args.v_cache.dtype != torch.uint8:
            raise ValueError("NVFP4 packed caches must be uint8")
        if args.k_scales is None or args.v_scales is None:
            raise ValueError("NVFP4 block scales are required")
        expected_cache = (args.k_cache.shape[0], DONOR_PAGE_SIZE, args.num_kv_heads, args.dim // 2)
        expected_scales = (args.k_cache.shape[0], DONOR_PAGE_SIZE, args.num_kv_heads, args.dim // 16)
        if tuple(args.k_cache.shape) != expected_cache or tuple(args.v_cache.shape) != expected_cache:
            raise ValueError(f"unexpected donor NVFP4 cache shape: {tuple(args.k_cache.shape)}")
        if tuple(args.k_scales.shape) != expected_scales or tuple(args.v_scales.shape) != expected_scales:
            raise ValueError(f"unexpected donor NVFP4 scale shape: {tuple(args.k_scales.shape)}")
        if not all(t.is_contiguous() for t in (args.k_cache, args.v_cache, args.k_scales, args.v_scales)):
            raise ValueError("zero-copy 256-to-64 repaging requires contiguous donor caches")
        if args.block_table.dtype != torch.int32 or args.cache_seqlens.dtype != torch.int32:
            raise ValueError("block table and pre-append lengths must be int32")
        if not args.block_table.is_contiguous():
            raise ValueError("flat-addressed table kernels require a contiguous block table")
        if args.k is None or args.v is None:
            raise ValueError("adapter requires current K/V so it can own exactly one append")
        append_len = args.k.shape[1]
        if (tuple(args.k.shape) != (args.bsz, append_len, args.num_kv_heads, args.dim)
                or tuple(args.v.shape) != tuple(args.k.shape) or append_len != args.q_len):
            raise ValueError("current K/V must match the actual query width")
        if args.block_table.shape[0] != args.bsz:
            raise ValueError("block table batch dimension mismatch")
        return append_len

    # ---------------------------------------------------------------- state
    def _layer_state(self, args) -> _LayerState:
        key = (id(args.k_cache), tuple(args.block_table.shape))
        state = self.layer_states.get(key)
        if state is None:
            while len(self.layer_states) >= 256:
                self.layer_states.pop(next(iter(self.layer_states)))
            state = _LayerState()
            self.layer_states[key] = state
        return state

    def _workspace(self, state: _LayerState, args, q_len: int):
        max_tokens = args.block_table.shape[1] * PAGE
        key = (q_len, str(args.q.device))
        ws = state.workspaces.get(key)
        if ws is None:
            if _capturing():
                raise RuntimeError("split workspace must exist before CUDA graph capture")
            splits = ops.default_splits(args.q.device, max_tokens, q_len)
            ws = (splits, *ops.split_workspace(args.q.device, q_len, splits))
            state.workspaces[key] = ws
        return ws

    def _output(self, state: _LayerState, args) -> torch.Tensor:
        out = state.outputs.get(args.q_len)
        if out is None or out.dtype != args.q.dtype or out.device != args.q.device:
            if _capturing():
                raise RuntimeError("attention output must exist before CUDA graph capture")
            out = torch.empty_like(args.q)
            state.outputs[args.q_len] = out
        return out

    # --------------------------------------------------------------- routes
    def _decode(self, args, state: _LayerState) -> torch.Tensor:
        """Append + split + combine (replaces _append + _xqa, xqa.py:356-554)."""
        splits, po, pml = self._workspace(state, args, args.q_len)
        out = self._output(state, args)
        ops.nvfp4_attend(args.q, args.k, args.v, args.k_cache, args.v_cache, args.k_scales,
                         args.v_scales, args.block_table, args.cache_seqlens, out, po, pml,
                         splits, float(args.sm_scale))
        return out

    def _prefill(self, args, state: _LayerState) -> torch.Tensor:
        """q_len > 8: one append, then one NVFP4 prefill launch over the
        pages (query position s sees keys j <= pre + s, lower-right causal as
        xqa.py:662); replaces the reference's gather -> FP16 -> FP8 -> PRIMS /
        SDPA staging (xqa.py:612-768)."""
        ops.nvfp4_append(args.k, args.v, args.k_cache, args.v_cache, args.k_scales,
                         args.v_scales, args.block_table, args.cache_seqlens)
        out = torch.empty_like(args.q) if not _capturing() else self._output(state, args)
        ops.nvfp4_prefill(args.q, args.k_cache, args.v_cache, args.k_scales, args.v_scales,
                          args.block_table, args.cache_seqlens, out, float(args.sm_scale))
        return out

    def _capture(self, state: _LayerState, args) -> _Graph:
        static_q = torch.zeros_like(args.q)
        static_k = torch.zeros_like(args.k)
        static_v = torch.zeros_like(args.v)
        static_seqlens = args.cache_seqlens.clone()
        # the live table, not zeros: warm-up appends must land in a mapped page
        static_table = args.block_table.clone()
        staged = args._replace(q=static_q, k=static_k, v=static_v, cache_seqlens=static_seqlens,
                               block_table=static_table)
        try:
            self._workspace(state, staged, args.q_len)
            self._output(state, staged)
            side = torch.cuda.Stream(device=args.q.device)
            side.wait_stream(torch.cuda.current_stream(args.q.device))
            with torch.cuda.stream(side):
                self._decode(staged, state)
            torch.cuda.current_stream(args.q.device).wait_stream(side)
            torch.cuda.synchronize(args.q.device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                output = self._decode(staged, state)
        except Exception:
            return _Graph(None, static_q, static_k, static_v, static_seqlens, static_table, None,
                          None, failed=True)
        return _Graph(graph, static_q, static_k, static_v, static_seqlens, static_table, output,
                      tuple(weakref.ref(t) for t in (args.k_cache, args.v_cache, args.k_scales,
                                                     args.v_scales)))

    def __call__(self, args):
        if args.k_scales is None:
            return None  # non-NVFP4 attention falls through (xqa.py:777-779)
        append_len = self._validate_nvfp4(args)
        if not args.q.is_cuda:
            raise ValueError("qwarz_b200 operators run on CUDA tensors only (no CPU fallback)")
        self.max_observed_query = max(self.max_observed_query, args.q_len)
        state = self._layer_state(args)
        if args.q_len > XQA_MAX_QUERY:
            out = self._prefill(args, state)
            self.append_calls += 1
            self.routes["prefill"] += 1
            self.query_rows["prefill"] += args.q_len
            return out
        if self.decode_graphs and not _capturing():
            key = (args.q_len, float(args.sm_scale), args.q.dtype)
            g = state.graphs.get(key)
            if g is not None and not g.matches(args):
                del state.graphs[key]
                state.graph_calls[key] = 0
                self.routes["graph_dropped"] += 1
                g = None
            if g is None:
                state.graph_calls[key] += 1
                if state.graph_calls[key] < self.XQA_GRAPH_WARMUPS:
                    out = self._decode(args, state)
                    self.append_calls += 1
                    self.routes["decode_eager"] += 1
                    self.query_rows["decode_eager"] += append_len
                    return out
                g = self._capture(state, args)
                state.graphs[key] = g
                self.routes["graph_failed" if g.failed else "graph_captured"] += 1
            if not g.failed and g.graph is not None:
                try:
                    g.static_q.copy_(args.q)
                    g.static_k.copy_(args.k)
                    g.static_v.copy_(args.v)
                    g.static_seqlens.copy_(args.cache_seqlens)
                    g.static_table.copy_(args.block_table)
                    g.graph.replay()
                except Exception:
                    del state.graphs[key]
                    state.graph_calls[key] = 0
                    self.routes["graph_error"] += 1
                else:
                    self.append_calls += 1
                    self.routes["decode_graph"] += 1
                    self.query_rows["decode_graph"] += append_len
                    return g.output
        out = self._decode(args, state)
        self.append_calls += 1
        self.routes["decode_eager"] += 1
        self.query_rows["decode_eager"] += append_len
        return out

    def diagnostics(self) -> dict[str, Any]:
        return {
            "mode": self.mode,
            "prefill": self.prefill,
            "contract": {
                "target_cache": "one-level NVFP4 global=1, donor NHD page256",
                "kernel_cache": "native 256-token pages (no repaging)",
                "input_lengths": "pre-append int32",
                "kernel_lengths": "post-append = pre-append + actual K rows (on device)",
                "append_owner": "selected adapter route exactly once",
                "short_query": "Q1..8",
                "prefill": "Q>8: one append, then the NVFP4 prefill kernel (tcgen05) over the pages",
            },
            "routes": dict(self.routes),
            "query_rows": dict(self.query_rows),
            "append_calls": self.append_calls,
            "max_observed_query": self.max_observed_query,
            "layer_states": len(self.layer_states),
        }


@contextmanager
def install(dispatch_list: list, adapter: NVFP4AttentionAdapter | None = None):
    """Prepend the adapter to a dispatcher candidate list and restore it on
    exit (xqa.py:909-920, where the list is ExLlamaV3 dispatch._fns_fp8)."""
    runtime = adapter if adapter is not None else NVFP4AttentionAdapter()
    original = list(dispatch_list)
    dispatch_list[:] = [runtime, *original]
    try:
        yield runtime
    finally:
        dispatch_list[:] = original


# ------------------------------------------------------ engine-level mirror
_ADAPTER: NVFP4AttentionAdapter | None = None
_BLOCK_TABLES: dict = {}
_BOUND_PAGES: int | None = None
_ZERO_LENS: dict = {}


def cache_seqlens(cache_len, device):
    """One int32 length; a tensor is already on device (attention.py:144-156)."""
    if isinstance(cache_len, int):
        if cache_len == 0:
            key = str(device)
            tensor = _ZERO_LENS.get(key)
            if tensor is None:
                tensor = torch.zeros(1, dtype=torch.int32, device=device)
                _ZERO_LENS[key] = tensor
            return tensor, 0
        return torch.tensor([cache_len], dtype=torch.int32, device=device), cache_len
    return cache_len, None


def empty_cache(pages: int = 1, device="cuda"):
    """NVFP4 one-level cache of `pages` 256-token pages (attention.py:159-167)."""
    packed = (pages, PAGE, KV_HEADS, HEAD_DIM // 2)
    scales = (pages, PAGE, KV_HEADS, HEAD_DIM // 16)
    return (
        torch.zeros(packed, dtype=torch.uint8, device=device),
        torch.zeros(packed, dtype=torch.uint8, device=device),
        torch.zeros(scales, dtype=torch.float8_e4m3fn, device=device),
        torch.zeros(scales, dtype=torch.float8_e4m3fn, device=device),
    )


def bind_table_pages(pages):
    """Publish only the first `pages` identity entries on the next attend
    (attention.py:175-183): the table width bounds the walked sequence."""
    global _BOUND_PAGES
    _BOUND_PAGES = pages


def _block_table(pages, device):
    key = (pages, str(device))
    table = _BLOCK_TABLES.get(key)
    if table is None:
        table = torch.arange(pages, dtype=torch.int32, device=device).view(1, pages)
        _BLOCK_TABLES[key] = table
    return table


def release_attention_plans():
    global _BOUND_PAGES
    _BOUND_PAGES = None
    if _ADAPTER is not None:
        _ADAPTER.layer_states.clear()


def adapter() -> NVFP4AttentionAdapter:
    global _ADAPTER
    if _ADAPTER is None:
        # nested graphs cannot record a graph launch: eager inside an outer
        # capture, as the reference engine does (attention.py:207-211)
        _ADAPTER = NVFP4AttentionAdapter(decode_graphs=False,
                                         query_dtypes=(torch.float16, torch.bfloat16))
    return _ADAPTER


def attend(q, k, v, cache, cache_len=0, block_table=None):
    """engine.forward.attention.attend (attention.py:203-250) on the B200 kernels.

    q [1, S, 24, 256], k/v [1, S, 4, 256] (the new rows), cache the 4-tuple of
    `empty_cache`, cache_len the pre-append length (int or int32 [1] device
    tensor).  Returns [1, S, 24, 256] in the adapter's persistent buffer.
    block_table (int32 [1, P], optional) replaces the engine's identity
    table, e.g. for a cache whose pages were allocated out of order.
    """
    runtime = adapter()
    k_cache, v_cache, k_scales, v_scales = cache
    seqlen = q.shape[1]
    pages = k_cache.shape[0]
    runtime._host_cache_len = cache_len if isinstance(cache_len, int) else None
    table = _block_table(pages, q.device) if block_table is None else block_table
    bound = _BOUND_PAGES
    if bound is not None and bound < table.shape[1]:
        table = table.narrow(1, 0, bound)
    args = AttnArgs(
        bsz=1, q_len=seqlen, num_q_heads=HEADS, dim=HEAD_DIM, kv_len=seqlen,
        num_kv_heads=KV_HEADS, q=q.contiguous(), k=k.contiguous(), v=v.contiguous(),
        k_cache=k_cache, v_cache=v_cache, causal=True, sm_scale=HEAD_DIM ** -0.5,
        cu_seqlens=None, max_seqlen=None, window_size=None, softcap=0.0, block_table=table,
        cache_seqlens=cache_seqlens(cache_len, q.device)[0], k_scales=k_scales,
        v_scales=v_scales)
    return runtime(args)
