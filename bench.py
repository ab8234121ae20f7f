"""Benchmark of the NVFP4-KV decode attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload auto|c3|c4|c5|all]

Default workload ("auto"): one decode step = q_len 1 attention over 16
attention layers, each with independent seeded NVFP4 KV of 65,536 tokens per
GPU (BASELINE config 2 at N=1).  At N > 1 the 16 sequences are 65,536*N
tokens long and sharded contiguously by pages (N=4 is the 262,144-token
native context of config 4): per layer every rank runs the shard split (the
owner of the new row's page appends it), then one kernel merges its splits
into an (m, l, O) record, stores it into every rank's buffer over NVLink peer
memory and LSE-combines all records (--exchange nccl: an NCCL all-gather and
a separate combine) — "scaling": "weak" (per-GPU work fixed).

value  = whole-job algorithmic HBM bytes per step / device step time (GB/s);
         per layer 1152*L + 2*(24*256*2) + 4*P + 1152 + 2*4*256*2 bytes.
e2e    = the same bytes through the C-ABI call a caller makes per layer
         (qwz_nvfp4_attend via qwarz_b200.ops; ShardedDecode.step at N > 1),
         with every step's Q/K/V copied in from pinned host memory and the
         outputs copied back, all inside the timed region.
roofline: the split kernel alone (graph of its 16 launches), CUDA events.
Inputs: synthetic, seeded, BF16 ~N(0,1) with 4 outlier channels x8 (K, V)
quantised to NVFP4 by the library's own writer; 16 layers x 75.5 MB of KV
rotate through the step, so every layer's pages are evicted from the 126 MB
L2 before they are read again.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HEADS, KV_HEADS, DIM, PAGE = 24, 4, 256, 256
LAYERS = 16
TOKENS_PER_GPU = 65536
METRIC = "NVFP4-KV decode attn µs/step & HBM GB/s vs ~8 TB/s, 64K–262K ctx, 1–8 B200"


def layer_bytes(L: int, q_len: int = 1, pages: int | None = None) -> int:
    """Algorithmic HBM bytes of one layer call (KV codes+scales, Q in, O out,
    table, append write, new K/V read)."""
    P = pages if pages is not None else math.ceil(L / PAGE)
    return 1152 * L + 2 * (q_len * HEADS * DIM * 2) + 4 * P + 1152 * q_len + 2 * q_len * KV_HEADS * DIM * 2


def peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every 10 ms."""

    REASONS = {
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "sw_power_cap": 0x4, "gpu_idle": 0x1,
    }

    def __init__(self, index: int):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
                mask = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        if self.nvml is not None:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.nvml is not None:
            self._stop.set()
            self.thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ------------------------------------------------------------------- data
def build_layer(ops, device, pages: int, tokens: int, seed: int, dtype=torch.bfloat16):
    """One layer's NVFP4 cache: `tokens` seeded K/V rows written by the
    library's writer into `pages` pages in a seed-permuted order."""
    g = torch.Generator(device=device).manual_seed(seed)
    perm = torch.randperm(pages, generator=g, device=device).to(torch.int32)
    cache = (torch.zeros(pages, PAGE, KV_HEADS, DIM // 2, dtype=torch.uint8, device=device),
             torch.zeros(pages, PAGE, KV_HEADS, DIM // 2, dtype=torch.uint8, device=device),
             torch.zeros(pages, PAGE, KV_HEADS, DIM // 16, dtype=torch.float8_e4m3fn, device=device),
             torch.zeros(pages, PAGE, KV_HEADS, DIM // 16, dtype=torch.float8_e4m3fn, device=device))
    outl = torch.randperm(DIM, generator=g, device=device)[:4]
    zero = torch.zeros(1, dtype=torch.int32, device=device)
    chunk = 16384
    for t0 in range(0, tokens, chunk):
        n = min(chunk, tokens - t0)
        k = torch.randn(n, KV_HEADS, DIM, generator=g, device=device)
        v = torch.randn(n, KV_HEADS, DIM, generator=g, device=device)
        k[..., outl] *= 8
        v[..., outl] *= 8
        start = torch.full((1,), t0, dtype=torch.int32, device=device)
        ops.nvfp4_append(k.to(dtype).contiguous(), v.to(dtype).contiguous(), *cache, perm, start)
    del zero
    return cache, perm


def cuda_time(fn, iters: int, stream) -> float:
    """Total milliseconds of `iters` calls of fn, CUDA events on `stream`."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(iters):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


# ------------------------------------------------------------- CPU oracle
def cpu_oracle_sample(layers_cpu, tokens: int, seconds: float = 15.0):
    """Time the oracle port (dequant gather + FP32 attention) on host cores
    over whole layers of the workload until ~`seconds` of CPU work."""
    from oracle import attention as oatt

    torch.set_num_threads(os.cpu_count() or 1)
    done, t0 = 0, time.perf_counter()
    while True:
        cache, table, q = layers_cpu[done % len(layers_cpu)]
        oatt.nvfp4_attention(q.float(), cache[0], cache[1], cache[2].view(torch.uint8),
                             cache[3].view(torch.uint8), table, tokens - 1)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 64:
            break
    per_layer_s = el / done
    return {
        "value": layer_bytes(tokens) / per_layer_s / 1e9,
        "unit": "GB/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"{done} layer call(s) of the {tokens}-token q_len=1 decode (NVFP4 dequant gather "
                  f"+ FP32 softmax attention, torch CPU), {el:.1f} s, {per_layer_s * 1e3:.1f} ms/layer",
    }


def cpu_layers_for_oracle(device_layers, queries, n: int):
    out = []
    for i in range(n):
        cache, table = device_layers[i]
        out.append((tuple(t.cpu() for t in cache), table.cpu(), queries[i].float().cpu()))
    return out


# -------------------------------------------------------------- our arm
def run_ours(args, rank: int, world: int, device) -> dict | None:
    from qwarz_b200 import build, ops, sharded

    build.build()
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    tokens_total = TOKENS_PER_GPU * world
    pages_total = tokens_total // PAGE
    shards = sharded.shard_pages(pages_total, world)
    shard = shards[rank]
    local_pages = shard.num_pages
    local_tokens = shard.tok_span
    dtype = torch.bfloat16

    layers = []
    for l in range(LAYERS):
        cache, perm = build_layer(ops, device, local_pages, local_tokens, seed=1000 * rank + l)
        layers.append((cache, perm))
    g = torch.Generator(device=device).manual_seed(4242)
    q = [torch.randn(1, 1, HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(LAYERS)]
    knew = [torch.randn(1, 1, KV_HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(LAYERS)]
    vnew = [torch.randn(1, 1, KV_HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(LAYERS)]
    out = [torch.empty(1, 1, HEADS, DIM, dtype=dtype, device=device) for _ in range(LAYERS)]
    pre = torch.tensor([tokens_total - 1], dtype=torch.int32, device=device)
    torch.cuda.synchronize()

    splits = ops.default_splits(device, local_tokens, 1)
    exchange = None
    if world == 1:
        po, pml = ops.split_workspace(device, 1, splits)

        def step():
            for l in range(LAYERS):
                cache, perm = layers[l]
                ops.nvfp4_attend(q[l], knew[l], vnew[l], *cache, perm, pre, out[l], po, pml, splits)

        def split_only():
            for l in range(LAYERS):
                cache, perm = layers[l]
                ops.attn_split(q[l], cache[0], cache[1], perm, pre, po, pml, cache[2], cache[3], splits)
    else:
        dec = sharded.ShardedDecode(shard, device, 1, splits, exchange=args.exchange)
        exchange = dec.exchange

        def step():
            for l in range(LAYERS):
                cache, perm = layers[l]
                dec.step(q[l], knew[l], vnew[l], cache, perm, pre, out[l])

        def split_only():
            for l in range(LAYERS):
                cache, perm = layers[l]
                dec.partial(q[l], cache, perm, pre)

    def capture(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        torch.cuda.synchronize()
        return graph

    graph = capture(step)
    split_graph = capture(split_only)

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[device.index])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        graph.replay()
    barrier()
    with ClockSampler(device.index) as clocks:
        t_ms = cuda_time(graph.replay, args.steps, torch.cuda.current_stream(device))
        barrier()
        t_split_ms = cuda_time(split_graph.replay, args.steps, torch.cuda.current_stream(device))
        barrier()
    ms_step = t_ms / args.steps
    split_ms_launch = t_split_ms / args.steps / LAYERS

    # ----- end to end through the public API, host copies inside the graph:
    # one pinned H2D of the step's inputs (q, k, v of every layer, one
    # buffer) and one D2H of the step's outputs, per-layer calls on views.
    per_in = HEADS * DIM + 2 * KV_HEADS * DIM
    host_in = torch.empty(LAYERS, per_in, dtype=dtype).pin_memory()
    for l in range(LAYERS):
        host_in[l].copy_(torch.cat([q[l].flatten(), knew[l].flatten(), vnew[l].flatten()]).cpu())
    host_out = torch.empty(LAYERS, HEADS * DIM, dtype=dtype).pin_memory()
    dev_in = torch.empty(LAYERS, per_in, dtype=dtype, device=device)
    dev_out = torch.empty(LAYERS, HEADS * DIM, dtype=dtype, device=device)
    dq = [dev_in[l, :HEADS * DIM].view(1, 1, HEADS, DIM) for l in range(LAYERS)]
    dk = [dev_in[l, HEADS * DIM:HEADS * DIM + KV_HEADS * DIM].view(1, 1, KV_HEADS, DIM) for l in range(LAYERS)]
    dv = [dev_in[l, HEADS * DIM + KV_HEADS * DIM:].view(1, 1, KV_HEADS, DIM) for l in range(LAYERS)]
    do = [dev_out[l].view(1, 1, HEADS, DIM) for l in range(LAYERS)]
    h2d = host_in.numel() * host_in.element_size()
    d2h = host_out.numel() * host_out.element_size()
    if world == 1:
        def e2e_step():
            dev_in.copy_(host_in, non_blocking=True)
            for l in range(LAYERS):
                cache, perm = layers[l]
                ops.nvfp4_attend(dq[l], dk[l], dv[l], *cache, perm, pre, do[l], po, pml, splits)
            host_out.copy_(dev_out, non_blocking=True)
    else:
        def e2e_step():
            dev_in.copy_(host_in, non_blocking=True)
            for l in range(LAYERS):
                cache, perm = layers[l]
                dec.step(dq[l], dk[l], dv[l], cache, perm, pre, do[l])
            host_out.copy_(dev_out, non_blocking=True)

    e2e_graph = capture(e2e_step)
    for _ in range(args.warmup):
        e2e_graph.replay()
    barrier()
    e2e_ms = cuda_time(e2e_graph.replay, args.steps, torch.cuda.current_stream(device)) / args.steps
    barrier()
    del e2e_graph

    # ----- aggregate over ranks
    bytes_rank = LAYERS * layer_bytes(local_tokens, 1, local_pages)
    if world > 1:
        t = torch.tensor([ms_step, split_ms_launch, e2e_ms], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_step, split_ms_launch, e2e_ms = float(t[0]), float(t[1]), float(t[2])
    del graph, split_graph
    if world > 1:
        torch.cuda.synchronize()
        barrier()  # every rank is done with the peer buffers before any rank frees its own
        dec.close()
    if rank != 0:
        return None

    total_bytes = bytes_rank * world
    pk, pk_kind = peaks()
    achieved = layer_bytes(local_tokens, 1, local_pages) / (split_ms_launch * 1e-3) / 1e9
    traffic = None
    tr_path = ROOT / "profiles" / "decode_traffic.json"
    if tr_path.exists():
        try:
            traffic = json.loads(tr_path.read_text()).get("bytes_per_launch")
        except Exception:
            traffic = None
    result = {
        "metric": METRIC,
        "value": total_bytes / (ms_step * 1e-3) / 1e9,
        "unit": "GB/s",
        "us_per_step": ms_step * 1e3,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 Q/K/V/O; NVFP4 (E2M1 + E4M3/16) KV; f16 tensor-core MMA, f32 softmax/accumulate",
        "data": "synthetic (seeded BF16 N(0,1) K/V with 4 outlier channels x8, NVFP4-quantised by "
                "the library writer; BF16 N(0,1) Q)",
        "config": {
            "workload": ("C2: decode q_len=1, 16 attention layers x 65,536 tokens NVFP4 KV "
                         "(256 pages of 256, seed-permuted tables), GQA 24/4 x 256"
                         if world == 1 else
                         f"weak-scaled C4: decode q_len=1, 16 layers x {tokens_total} tokens "
                         f"sharded over {world} GPUs ({TOKENS_PER_GPU} per GPU), (m,l,O) records "
                         + ("exchanged over NVLink peer memory inside the merge kernel"
                            if exchange == "peer" else "all-gathered by NCCL") + " + LSE combine"),
            "layers": LAYERS, "context_tokens": tokens_total, "tokens_per_gpu": local_tokens,
            "q_len": 1, "heads": "24q/4kv", "head_dim": DIM, "page": PAGE, "splits_per_head": splits,
            "l2": "inputs larger than L2: 16 layers x 75.5 MB KV rotate per step",
            "graph": "one CUDA graph per step",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "nvfp4_decode_kernel (split-K, one launch per layer)",
            "achieved": achieved,
            "peak": pk["hbm_gbs"],
            "peak_kind": pk_kind,
            "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"],
            "traffic": traffic,
            "us_per_launch": split_ms_launch * 1e3,
            "algorithmic_bytes_per_launch": layer_bytes(local_tokens, 1, local_pages),
        },
        "e2e": None if e2e_ms is None else {
            "value": total_bytes / (e2e_ms * 1e-3) / 1e9,
            "unit": "GB/s",
            "us_per_step": e2e_ms * 1e3,
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": ("qwz_nvfp4_attend (C ABI, via qwarz_b200.ops.nvfp4_attend) per layer" if world == 1 else
                    f"qwarz_b200.sharded.ShardedDecode.step per layer ({exchange} exchange inside)")
                   + "; one pinned H2D of the step's q/k/v and one D2H of its outputs; "
                     "captured in one CUDA graph, max over ranks",
        },
        # our kernels per timed step: split with fused append + combine (N=1);
        # append, split, partial combine, gathered combine (N>1); plus the
        # split-only roofline graph
        "gpu_launches": args.steps * LAYERS * (2 if world == 1 or exchange == "peer" else 4) + args.steps * LAYERS,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        sample = cpu_layers_for_oracle(layers, [t.view(1, HEADS, DIM) for t in q], 2)
        result["cpu_baseline"] = cpu_oracle_sample(sample, local_tokens, args.cpu_seconds)
    return result


# ------------------------------------------------- other BASELINE configs
def graph_time_ms(fn, warmup: int, steps: int, stream) -> float:
    for _ in range(max(3, warmup)):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    ms = cuda_time(graph.replay, steps, stream) / steps
    del graph
    return ms


def run_extra(args, device) -> dict:
    """C3 (MTP7 verify at 32K and 131K), C4 (262K on one GPU) and C5 (FP8
    draft, 6 steps in one CUDA graph); one JSON object with per-config
    device times and HBM fractions (not the driver's headline line)."""
    from qwarz_b200 import build, ops
    from qwarz_b200.draft_attention import DecodeAttention, shadow_write

    build.build()
    stream = torch.cuda.current_stream(device)
    pk, pk_kind = peaks()
    res = {"workload": args.workload, "peak_gbs": pk["hbm_gbs"], "peak_kind": pk_kind, "configs": {}}
    g = torch.Generator(device=device).manual_seed(7)
    dtype = torch.bfloat16

    def nvfp4_config(tokens, q_len, layers):
        pages = tokens // PAGE
        lay = [build_layer(ops, device, pages, tokens, seed=3000 + l) for l in range(layers)]
        q = [torch.randn(q_len, HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(layers)]
        kn = [torch.randn(q_len, KV_HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(layers)]
        vn = [torch.randn(q_len, KV_HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(layers)]
        out = [torch.empty_like(t) for t in q]
        pre = torch.tensor([tokens - q_len], dtype=torch.int32, device=device)
        splits = ops.default_splits(device, tokens, q_len)
        po, pml = ops.split_workspace(device, q_len, splits)

        def step():
            for l in range(layers):
                c, perm = lay[l]
                ops.nvfp4_attend(q[l], kn[l], vn[l], *c, perm, pre, out[l], po, pml, splits)

        def split_only():
            for l in range(layers):
                c, perm = lay[l]
                ops.attn_split(q[l], c[0], c[1], perm, pre, po, pml, c[2], c[3], splits)

        ms = graph_time_ms(step, args.warmup, args.steps, stream)
        ms_split = graph_time_ms(split_only, args.warmup, args.steps, stream) / layers
        byt = layer_bytes(tokens, q_len, pages)
        del lay
        torch.cuda.empty_cache()
        return {"tokens": tokens, "q_len": q_len, "layers": layers, "splits": splits,
                "us_per_step": ms * 1e3, "us_per_layer_call": ms * 1e3 / layers,
                "split_us_per_launch": ms_split * 1e3,
                "split_GBps": byt / (ms_split * 1e-3) / 1e9,
                "split_frac": byt / (ms_split * 1e-3) / 1e9 / pk["hbm_gbs"],
                "step_GBps": layers * byt / (ms * 1e-3) / 1e9,
                "verify_flops_per_layer": 4 * 256 * 24 * (q_len * (tokens - q_len) + q_len * (q_len + 1) // 2)}

    if args.workload in ("c3", "all"):
        for tokens in (32768, 131072):
            v7 = nvfp4_config(tokens, 7, 16)
            d1 = nvfp4_config(tokens, 1, 16)
            v7["tensor_TFLOPs_split"] = v7["verify_flops_per_layer"] / (v7["split_us_per_launch"] * 1e-6) / 1e12
            res["configs"][f"c3_{tokens}"] = {"verify_q7": v7, "decode_q1": d1,
                                              "verify_over_decode_step": v7["us_per_step"] / d1["us_per_step"]}
    if args.workload in ("prefill", "all"):
        # NVFP4 prefill (SURVEY next item 1): one launch over the pages vs the
        # 8-row-window route through the verify kernel it replaces
        for pre, S in ((0, 8192), (61440, 4096)):
            tokens = pre + S
            pages = (tokens + PAGE - 1) // PAGE
            c, perm = build_layer(ops, device, pages, tokens, seed=5000 + S)
            q = torch.randn(S, HEADS, DIM, generator=g, device=device).to(dtype)
            out = torch.empty_like(q)
            pre_t = torch.tensor([pre], dtype=torch.int32, device=device)

            def prefill():
                ops.nvfp4_prefill(q, c[0], c[1], c[2], c[3], perm, pre_t, out)

            splits = ops.default_splits(device, tokens, 8)
            po, pml = ops.split_workspace(device, 8, splits)
            wl = torch.arange(pre, pre + S, 8, dtype=torch.int32, device=device)

            def windows():
                for w in range(S // 8):
                    ops.attn_split(q[8 * w:8 * w + 8], c[0], c[1], perm, wl[w:w + 1], po, pml, c[2], c[3], splits)
                    ops.attn_combine(po, pml, out[8 * w:8 * w + 8], splits)

            for _ in range(2):
                prefill()
            ms = cuda_time(prefill, 5, stream) / 5
            ms_w = graph_time_ms(windows, 1, 2, stream)  # the old route, graph-captured
            flops = 4 * HEADS * DIM * sum(pre + s + 1 for s in range(S))
            res["configs"][f"prefill_{pre}+{S}"] = {
                "pre": pre, "q_len": S, "us_per_layer": ms * 1e3, "TFLOPs": flops / (ms * 1e-3) / 1e12,
                "tensor_frac_of_measured_bf16": flops / (ms * 1e-3) / 1e12 / pk.get("bf16_tflops", 1590.0),
                "windowed_verify_us": ms_w * 1e3, "speedup_vs_windows": ms_w / ms}
            del c, perm
            torch.cuda.empty_cache()
        # draft-model prefill (SURVEY next item 3): FP16 K/V read in place vs
        # the reference's torch route for the same shapes (draft.py:33-86:
        # SDPA causal when S == T, else the LSE merge of two flash calls)
        from qwarz_b200.draft_attention import draft_attend
        for pre, S in ((0, 8192), (61440, 4096)):
            T = pre + S
            qd = torch.randn(1, S, HEADS, DIM, generator=g, device=device).half()
            kd = torch.randn(1, T, KV_HEADS, DIM, generator=g, device=device).half()
            vd = torch.randn(1, T, KV_HEADS, DIM, generator=g, device=device).half()
            outd = torch.empty_like(qd)

            def ours():
                ops.draft_prefill(qd, kd, vd, outd, DIM ** -0.5)

            expand = [False]  # GQA through the flash op, else heads repeated first

            def sdpa_route():
                qt, kt, vt = qd.transpose(1, 2), kd.transpose(1, 2), vd.transpose(1, 2)
                if pre == 0:
                    o = torch.nn.functional.scaled_dot_product_attention(
                        qt, kt, vt, is_causal=True, scale=DIM ** -0.5, enable_gqa=True)
                else:
                    if expand[0]:
                        kt = kt.repeat_interleave(HEADS // KV_HEADS, 1)
                        vt = vt.repeat_interleave(HEADS // KV_HEADS, 1)
                    op = torch.ops.aten._scaled_dot_product_flash_attention
                    o1, l1, *_ = op(qt, kt[:, :, :pre], vt[:, :, :pre], 0.0, False, False, scale=DIM ** -0.5)
                    o2, l2, *_ = op(qt, kt[:, :, pre:], vt[:, :, pre:], 0.0, True, False, scale=DIM ** -0.5)
                    a, b = l1.unsqueeze(-1), l2.unsqueeze(-1)
                    tot = torch.logaddexp(a, b)
                    o = (o1.float() * (a - tot).exp() + o2.float() * (b - tot).exp()).half()
                return o.transpose(1, 2).contiguous()

            for _ in range(2):
                ours()
            ms = cuda_time(ours, 5, stream) / 5
            try:
                sdpa_route()
            except RuntimeError:
                expand[0] = True
            for _ in range(2):
                sdpa_route()
            ms_ref = cuda_time(sdpa_route, 3, stream) / 3
            flops = 4 * HEADS * DIM * sum(pre + s + 1 for s in range(S))
            res["configs"][f"draft_prefill_{pre}+{S}"] = {
                "pre": pre, "q_len": S, "us_per_layer": ms * 1e3, "TFLOPs": flops / (ms * 1e-3) / 1e12,
                "tensor_frac_of_measured_bf16": flops / (ms * 1e-3) / 1e12 / pk.get("bf16_tflops", 1590.0),
                "torch_sdpa_route_us": ms_ref * 1e3, "sdpa_heads_repeated": expand[0],
                "speedup_vs_sdpa_route": ms_ref / ms}
            del qd, kd, vd, outd
            torch.cuda.empty_cache()
    if args.workload in ("c4", "all"):
        res["configs"]["c4_262144_1gpu"] = nvfp4_config(262144, 1, 16)
    if args.workload in ("c5", "all"):
        T = 65536 + 6
        base = 65536
        kf = torch.randn(T, KV_HEADS, DIM, generator=g, device=device)
        vf = torch.randn(T, KV_HEADS, DIM, generator=g, device=device)
        pages = (T + PAGE - 1) // PAGE
        ksc = torch.full((pages, KV_HEADS), 0.02, dtype=torch.float32, device=device)
        vsc = torch.full((pages, KV_HEADS), 0.03, dtype=torch.float32, device=device)
        k8 = (kf / 0.02).clamp(-448, 448).to(torch.float8_e4m3fn)[None]
        v8 = (vf / 0.03).clamp(-448, 448).to(torch.float8_e4m3fn)[None]
        del kf, vf
        attn = DecodeAttention(HEADS, KV_HEADS, DIM, device)
        qd = torch.randn(1, 1, HEADS, DIM, generator=g, device=device).half()
        kn = torch.randn(6, KV_HEADS, DIM, generator=g, device=device).half()
        vn = torch.randn(6, KV_HEADS, DIM, generator=g, device=device).half()
        outd = torch.empty_like(qd)
        pos = [torch.tensor([base + i], dtype=torch.int32, device=device) for i in range(6)]
        lens = [torch.tensor([base + i + 1], dtype=torch.int32, device=device) for i in range(6)]

        def roll():  # the shadow write fused into the draft kernel: two launches per step
            for i in range(6):
                attn.step(qd, kn[i], vn[i], k8, v8, pos[i], lens[i], outd, ksc, vsc)

        def roll_unfused():  # write kernel, draft kernel, combine
            for i in range(6):
                shadow_write(kn[i], vn[i], k8[0], v8[0], pos[i], ksc, vsc)
                attn.attend(qd, k8, v8, lens[i], outd, ksc, vsc)

        ms_unfused = graph_time_ms(roll_unfused, args.warmup, args.steps, stream)
        ms = graph_time_ms(roll, args.warmup, args.steps, stream)
        step_bytes = 2 * 4 * 256 * (base + 3) + 2 * 4 * 4 * pages + 2 * 24 * 256 * 2 + 2 * 4 * 256 * 3
        res["configs"]["c5_draft_fp8"] = {
            "tokens": base, "steps_per_graph": 6, "splits": attn.splits, "us_per_graph": ms * 1e3,
            "us_per_step": ms * 1e3 / 6, "us_per_step_unfused_write": ms_unfused * 1e3 / 6, "GBps": 6 * step_bytes / (ms * 1e-3) / 1e9,
            "frac": 6 * step_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"]}
    return res


def run_profile_case(args, device) -> dict:
    """Small case for ncu --set full: one 65,536-token layer (75.5 MB, above
    the L2 working set only with ncu's cache flush between passes), three
    eager launches of the decode split, the q_len 7 verify split, or the FP8
    draft decode."""
    from qwarz_b200 import build, ops
    from qwarz_b200.draft_attention import DecodeAttention

    build.build()
    tokens, pages = 65536, 256
    g = torch.Generator(device=device).manual_seed(11)
    if args.workload == "profile_prefill":
        # one NVFP4 prefill (8,192 rows onto an empty cache) then one draft
        # prefill of the same shape: 9.4 MB of pages, 100 MB of Q and of O
        S = 8192
        cache, perm = build_layer(ops, device, S // PAGE, S, seed=2)
        q = torch.randn(S, HEADS, DIM, generator=g, device=device).bfloat16()
        out = torch.empty_like(q)
        pre = torch.zeros(1, dtype=torch.int32, device=device)
        ops.nvfp4_prefill(q, cache[0], cache[1], cache[2], cache[3], perm, pre, out)
        qd = q.half()[None]
        kd = torch.randn(1, S, KV_HEADS, DIM, generator=g, device=device).half()
        vd = torch.randn(1, S, KV_HEADS, DIM, generator=g, device=device).half()
        ops.draft_prefill(qd, kd, vd, torch.empty_like(qd))
        torch.cuda.synchronize()
        return {"workload": args.workload, "tokens": S, "ok": True}
    if args.workload == "profile_draft":
        T = tokens + 6
        k8 = torch.randn(1, T, KV_HEADS, DIM, generator=g, device=device).to(torch.float8_e4m3fn)
        v8 = torch.randn(1, T, KV_HEADS, DIM, generator=g, device=device).to(torch.float8_e4m3fn)
        q = torch.randn(1, 1, HEADS, DIM, generator=g, device=device).half()
        out = torch.empty_like(q)
        attn = DecodeAttention(HEADS, KV_HEADS, DIM, device)
        length = torch.tensor([tokens], dtype=torch.int32, device=device)
        for _ in range(3):
            attn.attend(q, k8, v8, length, out)
    else:
        q_len = 7 if args.workload == "profile_verify" else 1
        cache, perm = build_layer(ops, device, pages, tokens, seed=1)
        q = torch.randn(q_len, HEADS, DIM, generator=g, device=device).bfloat16()
        pre = torch.tensor([tokens - q_len], dtype=torch.int32, device=device)
        splits = ops.default_splits(device, tokens, q_len)
        po, pml = ops.split_workspace(device, q_len, splits)
        out = torch.empty_like(q)
        for _ in range(3):
            ops.attn_split(q, cache[0], cache[1], perm, pre, po, pml, cache[2], cache[3], splits)
            ops.attn_combine(po, pml, out, splits)
    torch.cuda.synchronize()
    return {"workload": args.workload, "tokens": tokens, "ok": True}


# --------------------------------------------------------- reference arm
def run_reference(args) -> dict:
    """The reference's CPU oracle path, restated (oracle/), on host cores:
    NVFP4 -> dequant gather (xqa.py:73-143) + FP32 softmax attention
    (xqa.py:612-673), one 65,536-token layer call per step."""
    import numpy as np
    from oracle import attention as oatt
    from oracle import nvfp4
    from tests.golden import cases

    torch.set_num_threads(os.cpu_count() or 1)
    tokens = TOKENS_PER_GPU
    pages = tokens // PAGE
    layers = []
    for l in range(2):
        k = cases.kv_rows(900 + l, tokens)
        v = cases.kv_rows(950 + l, tokens)
        kc, ks = nvfp4.quantize_rows(k)
        vc, vs = nvfp4.quantize_rows(v)
        perm = np.random.default_rng(l).permutation(pages).astype(np.int32)
        inv = np.empty_like(perm)
        inv[perm] = np.arange(pages, dtype=np.int32)
        def paged(a):
            a = a.reshape(pages, PAGE, *a.shape[1:])
            return torch.from_numpy(np.ascontiguousarray(a[inv]))
        q = torch.randn(1, HEADS, DIM, generator=torch.Generator().manual_seed(l)).bfloat16()
        layers.append(((paged(kc), paged(vc), paged(ks), paged(vs)), torch.from_numpy(perm), q))

    def one(i):
        cache, table, q = layers[i % len(layers)]
        oatt.nvfp4_attention(q.float(), cache[0], cache[1], cache[2], cache[3], table, tokens - 1)

    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one(i)
    el = time.perf_counter() - t0
    per = el / args.steps
    value = layer_bytes(tokens) / per / 1e9
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "us_per_step": per * 1e6 * LAYERS,
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per * 1e3 * LAYERS,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "NVFP4 KV dequantised to FP32; FP32 softmax attention",
        "data": "synthetic (seeded N(0,1) K/V with 4 outlier channels x8, NVFP4 by the oracle writer)",
        "config": {"workload": "C2 sample: one 65,536-token q_len=1 decode layer call per step "
                               "(ms_per_step scaled to 16 layers)",
                   "layers_timed_per_step": 1, "context_tokens": tokens},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{args.steps} layer calls after {args.warmup} warm-up, "
                                   f"{per * 1e3:.1f} ms per layer call"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="auto", choices=["auto", "peer", "nccl"],
                    help="N>1: exchange of the shard records (auto: NVLink peer memory when every "
                         "rank can reach every GPU, else NCCL)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--workload", default="auto",
                    choices=["auto", "c3", "c4", "c5", "prefill", "all", "profile_prefill", "profile_decode",
                             "profile_verify", "profile_draft"],
                    help="auto: the driver's headline (C2 at N=1, weak-scaled sharding at N>1); "
                         "c3/c4/c5/all: the other BASELINE configs on one GPU (separate JSON); "
                         "profile_*: three eager launches of one kernel on one 65,536-token layer, "
                         "the small case for ncu --set full")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(run_reference(args)), flush=True)
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.workload.startswith("profile_"):
        print(json.dumps(run_profile_case(args, device)), flush=True)
        return
    if args.workload != "auto":
        print(json.dumps(run_extra(args, device)), flush=True)
        return
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    try:
        result = run_ours(args, rank, world, device)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
