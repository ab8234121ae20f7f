"""Benchmark of the NVFP4-KV decode attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload auto|c3|c4|c5|k8v4|prefill|all|profile_*]

Default workload ("auto"):

N = 1   BASELINE config 2.  One step is q_len 1 decode attention over 16
        attention layers, each with independent seeded NVFP4 KV of 65,536
        tokens.  The line also carries sub-records of the other single-GPU
        configs: the MTP7 verify at 32,768 and 131,072 tokens beside the
        decode at the same contexts (config 3), 262,144 tokens on one GPU
        (config 4), the FP8 draft, six steps in one CUDA graph, at the 16
        chunks the config names (config 5), the K8/V4 slot (decode at 65,536
        tokens, verify at 32,768 and 131,072) and the two prefill kernels
        (NVFP4 pages and the draft model's FP16 rows).
N > 1   BASELINE config 4, strong scaling.  16 layers of one 262,144-token
        sequence, its 1,024 pages split contiguously over the N GPUs.  Per
        layer every rank runs the shard split (the rank whose pages hold the
        new row appends it inside its decode kernel), then one kernel merges
        the rank's splits into an (m, l, O) record, stores it into every
        rank's buffer over NVLink peer memory and LSE-combines all records
        (--exchange nccl: an NCCL all-gather and a separate combine).  Before
        each timed window every rank replays the step once more, untimed: its
        exchange kernels finish only when every rank has reached them, so the
        ranks' start events fire together.  The line carries each rank's time
        (the reported one is the max), the split kernel alone, the exchange
        alone, the same 16-layer 262,144-token step on rank 0's GPU alone, and
        a check: every rank's output is bit-identical, and rank 0's equals the
        one-GPU output of the same layer within the parity tolerance.

value  = whole-job algorithmic HBM bytes per step / device step time (GB/s);
         per layer call 1152*L + 2*(24*256*2) + 4*P + 1152 + 2*4*256*2 bytes.
e2e    = the same bytes through the public API a caller uses, with every
         step's Q/K/V copied in from pinned host memory and the outputs copied
         back inside the timed region: qwarz_b200.attention.attend per layer
         (N = 1), captured in the caller's CUDA graph as the engine does;
         ShardedDecode.step per layer (N > 1).
roofline: the split kernel alone (a graph of its 16 launches), CUDA events.
Inputs: synthetic, seeded, BF16 ~N(0,1) with 4 outlier channels x8 (K, V)
quantised to NVFP4 by the library's own writer.  The layers of a step (16 x
75.5 MB at N = 1) rotate past the 126 MB L2, so a layer's pages are evicted
before they are read again.
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
C2_TOKENS = 65536
C4_TOKENS = 262144
ROW_CHUNK = 16384  # K/V rows are generated per aligned chunk of logical positions
METRIC = "NVFP4-KV decode attn µs/step & HBM GB/s vs ~8 TB/s, 64K–262K ctx, 1–8 B200"
DATA = ("synthetic (seeded BF16 N(0,1) K/V with 4 outlier channels x8, NVFP4-quantised by "
        "the library writer; BF16 N(0,1) Q)")
DTYPE = "bf16 Q/K/V/O; NVFP4 (E2M1 + E4M3/16) KV; f16 tensor-core MMA, f32 softmax/accumulate"


def layer_bytes(L: int, q_len: int = 1, pages: int | None = None) -> int:
    """Algorithmic HBM bytes of one layer call (KV codes+scales, Q in, O out,
    table, append write, new K/V read)."""
    P = pages if pages is not None else math.ceil(L / PAGE)
    return 1152 * L + 2 * (q_len * HEADS * DIM * 2) + 4 * P + 1152 * q_len + 2 * q_len * KV_HEADS * DIM * 2


def draft_step_bytes(L: int) -> int:
    """Algorithmic bytes of one FP8 draft step over L attended keys: K and V
    E4M3, the per-page-per-head FP32 scales, Q in and O out (FP16), and the
    new row's FP16 K/V read and E4M3 write (the fused shadow write)."""
    return (2 * KV_HEADS * DIM * L + 2 * KV_HEADS * 4 * math.ceil(L / PAGE) + 2 * HEADS * DIM * 2
            + 2 * KV_HEADS * DIM * (2 + 1))


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
def _chunk_rows(seed: int, chunk: int, device, outl):
    """K and V rows of the ROW_CHUNK logical positions of chunk `chunk`
    (seeded by layer seed and chunk only, so a shard of a sequence and the
    whole sequence hold the same rows)."""
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + chunk)
    k = torch.randn(ROW_CHUNK, KV_HEADS, DIM, generator=g, device=device)
    v = torch.randn(ROW_CHUNK, KV_HEADS, DIM, generator=g, device=device)
    k[..., outl] *= 8
    v[..., outl] *= 8
    return k, v


def build_layer(ops, device, pages: int, tokens: int, seed: int, first_token: int = 0,
                perm_seed: int | None = None, dtype=torch.bfloat16):
    """One layer's NVFP4 cache: the K/V rows of logical positions
    [first_token, first_token + tokens), written by the library's writer
    into `pages` pages in a seed-permuted physical order.  Returns
    (cache 4-tuple, block table [pages] int32)."""
    gp = torch.Generator(device=device).manual_seed(perm_seed if perm_seed is not None else 7919 * seed + 17)
    perm = torch.randperm(pages, generator=gp, device=device).to(torch.int32)
    go = torch.Generator(device=device).manual_seed(seed)
    outl = torch.randperm(DIM, generator=go, device=device)[:4]
    cache = (torch.zeros(pages, PAGE, KV_HEADS, DIM // 2, dtype=torch.uint8, device=device),
             torch.zeros(pages, PAGE, KV_HEADS, DIM // 2, dtype=torch.uint8, device=device),
             torch.zeros(pages, PAGE, KV_HEADS, DIM // 16, dtype=torch.float8_e4m3fn, device=device),
             torch.zeros(pages, PAGE, KV_HEADS, DIM // 16, dtype=torch.float8_e4m3fn, device=device))
    pos = first_token
    end = first_token + tokens
    while pos < end:
        chunk = pos // ROW_CHUNK
        lo = pos - chunk * ROW_CHUNK
        n = min(ROW_CHUNK - lo, end - pos)
        k, v = _chunk_rows(seed, chunk, device, outl)
        start = torch.full((1,), pos - first_token, dtype=torch.int32, device=device)
        ops.nvfp4_append(k[lo:lo + n].to(dtype).contiguous(), v[lo:lo + n].to(dtype).contiguous(),
                         *cache, perm, start)
        pos += n
    return cache, perm


def new_rows(device, layers: int, q_len: int = 1, dtype=torch.bfloat16):
    """Per-layer q [q_len, 24, 256] and new K/V rows [q_len, 4, 256] (the same
    on every rank: one seeded generator per device)."""
    g = torch.Generator(device=device).manual_seed(4242)
    q = [torch.randn(1, q_len, HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(layers)]
    k = [torch.randn(1, q_len, KV_HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(layers)]
    v = [torch.randn(1, q_len, KV_HEADS, DIM, generator=g, device=device).to(dtype) for _ in range(layers)]
    return q, k, v


# ----------------------------------------------------------------- timing
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


def capture(fn, warmup: int):
    """Run fn eagerly max(3, warmup) times, then capture it in a CUDA graph."""
    for _ in range(max(3, warmup)):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    torch.cuda.synchronize()
    return graph


def graph_ms(fn, warmup: int, steps: int, stream) -> float:
    """Milliseconds per replay of fn captured in one CUDA graph."""
    graph = capture(fn, warmup)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    ms = cuda_time(graph.replay, steps, stream) / steps
    del graph
    return ms


def ulp_bf16(x: torch.Tensor) -> torch.Tensor:
    """One unit in the last place of BF16 at |x|."""
    e = torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -126)))
    return torch.ldexp(torch.ones_like(x), (e - 7).to(torch.int32))


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


# ---------------------------------------------------- single-GPU configs
def nvfp4_config(ops, device, stream, args, pk, tokens: int, layers: int, q_lens=(1,), seed0: int = 3000):
    """Decode (q_len 1) and/or verify (q_len 7) over `layers` independent
    NVFP4 layers of `tokens` tokens: per q_len the split kernel alone and the
    whole layer call (append + split + combine), each a graph of `layers`
    launches or calls."""
    pages = tokens // PAGE
    lay = [build_layer(ops, device, pages, tokens, seed=seed0 + l) for l in range(layers)]
    res = {}
    for q_len in q_lens:
        q, kn, vn = new_rows(device, layers, q_len)
        q = [t.view(q_len, HEADS, DIM) for t in q]
        kn = [t.view(q_len, KV_HEADS, DIM) for t in kn]
        vn = [t.view(q_len, KV_HEADS, DIM) for t in vn]
        out = [torch.empty_like(t) for t in q]
        pre = torch.tensor([tokens - q_len], dtype=torch.int32, device=device)
        splits = ops.default_splits(device, tokens, q_len)
        po, pml = ops.split_workspace(device, q_len, splits)

        def call():
            for l in range(layers):
                c, perm = lay[l]
                ops.nvfp4_attend(q[l], kn[l], vn[l], *c, perm, pre, out[l], po, pml, splits)

        def split_only():
            for l in range(layers):
                c, perm = lay[l]
                ops.attn_split(q[l], c[0], c[1], perm, pre, po, pml, c[2], c[3], splits)

        ms_call = graph_ms(call, args.warmup, args.steps, stream) / layers
        ms_split = graph_ms(split_only, args.warmup, args.steps, stream) / layers
        byt = layer_bytes(tokens, q_len, pages)
        r = {"tokens": tokens, "q_len": q_len, "layers_rotated": layers, "splits": splits,
             "algorithmic_bytes_per_launch": byt,
             "split_us_per_launch": ms_split * 1e3,
             "split_GBps": byt / (ms_split * 1e-3) / 1e9,
             "split_frac": byt / (ms_split * 1e-3) / 1e9 / pk["hbm_gbs"],
             "call_us_per_layer": ms_call * 1e3,
             "call_GBps": byt / (ms_call * 1e-3) / 1e9}
        if q_len > 1:
            flops = 4 * DIM * HEADS * (q_len * (tokens - q_len) + q_len * (q_len + 1) // 2)
            r["flops_per_launch"] = flops
            r["split_TFLOPs"] = flops / (ms_split * 1e-3) / 1e12
        res[f"q{q_len}"] = r
    del lay
    torch.cuda.empty_cache()
    return res


def c3_record(ops, device, stream, args, pk):
    """Config 3: MTP7 verify beside the decode at the same context."""
    out = {}
    for tokens, layers in ((32768, 8), (131072, 4)):
        r = nvfp4_config(ops, device, stream, args, pk, tokens, layers, q_lens=(7, 1))
        r["verify_over_decode_split"] = r["q7"]["split_us_per_launch"] / r["q1"]["split_us_per_launch"]
        r["verify_over_decode_call"] = r["q7"]["call_us_per_layer"] / r["q1"]["call_us_per_layer"]
        out[str(tokens)] = r
    return out


def c5_record(device, stream, args, pk, splits_list=(16, 37)):
    """Config 5: six sequential FP8 draft steps (shadow write fused) over
    65,536 + 6 slots with per-page-per-head scales, in one CUDA graph."""
    from qwarz_b200.draft_attention import DecodeAttention

    base = C2_TOKENS
    T = base + 6
    g = torch.Generator(device=device).manual_seed(7)
    pages = (T + PAGE - 1) // PAGE
    ksc = torch.full((pages, KV_HEADS), 0.02, dtype=torch.float32, device=device)
    vsc = torch.full((pages, KV_HEADS), 0.03, dtype=torch.float32, device=device)
    k8 = (torch.randn(T, KV_HEADS, DIM, generator=g, device=device) / 0.02).clamp(-448, 448).to(torch.float8_e4m3fn)[None]
    v8 = (torch.randn(T, KV_HEADS, DIM, generator=g, device=device) / 0.03).clamp(-448, 448).to(torch.float8_e4m3fn)[None]
    qd = torch.randn(1, 1, HEADS, DIM, generator=g, device=device).half()
    kn = torch.randn(6, KV_HEADS, DIM, generator=g, device=device).half()
    vn = torch.randn(6, KV_HEADS, DIM, generator=g, device=device).half()
    outd = torch.empty_like(qd)
    pos = [torch.tensor([base + i], dtype=torch.int32, device=device) for i in range(6)]
    lens = [torch.tensor([base + i + 1], dtype=torch.int32, device=device) for i in range(6)]
    step_bytes = sum(draft_step_bytes(base + i + 1) for i in range(6)) / 6
    res = {}
    for splits in splits_list:
        attn = DecodeAttention(HEADS, KV_HEADS, DIM, device, splits=splits)

        def roll():
            for i in range(6):
                attn.step(qd, kn[i], vn[i], k8, v8, pos[i], lens[i], outd, ksc, vsc)

        ms = graph_ms(roll, args.warmup, args.steps, stream)
        res[f"splits_{splits}"] = {"splits": splits, "us_per_graph": ms * 1e3, "us_per_step": ms * 1e3 / 6,
                                   "GBps": 6 * step_bytes / (ms * 1e-3) / 1e9,
                                   "frac": 6 * step_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"]}
    res["tokens"] = base
    res["baseline_chunks"] = 16
    return res


K8V4_TOKEN_BYTES = 1664  # K 1,024 + V 512 + 2 x 64 B of FP16 scales per token (4 KV heads)


def k8v4_layer(device, pages: int, tokens: int, seed: int):
    """One K8/V4 layer of `tokens` seeded BF16 rows (4 outlier channels x8),
    quantised by the library's writer into `pages` pages in a seed-permuted
    order.  Returns (cache 4-tuple, block table)."""
    from qwarz_b200 import k8v4

    cache = k8v4.empty_cache(pages, device)
    g = torch.Generator(device=device).manual_seed(seed)
    perm = torch.randperm(pages, generator=g, device=device).to(torch.int32)
    outl = torch.randperm(DIM, generator=g, device=device)[:4]
    for t0 in range(0, tokens, 16384):
        n = min(16384, tokens - t0)
        k = torch.randn(n, KV_HEADS, DIM, generator=g, device=device)
        v = torch.randn(n, KV_HEADS, DIM, generator=g, device=device)
        k[..., outl] *= 8.0
        v[..., outl] *= 8.0
        start = torch.tensor([t0], dtype=torch.int32, device=device)
        k8v4.append(k.bfloat16(), v.bfloat16(), cache, perm, start)
    return cache, perm


def k8v4_record(device, stream, args, pk):
    """The K8/V4 cache path (the reference's Attention64 split/combine slot):
    decode at 65,536 tokens and MTP7 verify at 32,768 / 131,072, split alone
    and split + rotating combine per layer, rotating over layers so the
    pages exceed L2.  Algorithmic bytes: 1,664 B per token plus the table."""
    from qwarz_b200 import k8v4, ops

    res = {"token_bytes": K8V4_TOKEN_BYTES}
    h32 = k8v4.hadamard32(device)
    for tokens, layers, q_len in ((65536, 4, 1), (32768, 8, 7), (131072, 2, 7)):
        pages = tokens // PAGE
        lay = [k8v4_layer(device, pages, tokens, 9000 + l) for l in range(layers)]
        g = torch.Generator(device=device).manual_seed(77)
        q = [torch.randn(q_len, HEADS, DIM, generator=g, device=device).bfloat16() for _ in range(layers)]
        out = [torch.empty_like(t) for t in q]
        pre = torch.tensor([tokens - q_len], dtype=torch.int32, device=device)
        splits = ops.default_splits(device, tokens, q_len)
        po, pml = ops.split_workspace(device, q_len, splits)

        def split_only():
            for l in range(layers):
                k8v4.split(q[l], lay[l][0], lay[l][1], pre, po, pml, h32, splits)

        def call():
            for l in range(layers):
                k8v4.split(q[l], lay[l][0], lay[l][1], pre, po, pml, h32, splits)
                k8v4.combine(po, pml, out[l], h32, splits)

        ms_split = graph_ms(split_only, args.warmup, args.steps, stream) / layers
        ms_call = graph_ms(call, args.warmup, args.steps, stream) / layers
        byt = tokens * K8V4_TOKEN_BYTES + 4 * pages
        res[f"{tokens}_q{q_len}"] = {
            "tokens": tokens, "q_len": q_len, "layers_rotated": layers, "splits": splits,
            "algorithmic_bytes_per_launch": byt, "split_us_per_launch": ms_split * 1e3,
            "split_GBps": byt / (ms_split * 1e-3) / 1e9, "split_frac": byt / (ms_split * 1e-3) / 1e9 / pk["hbm_gbs"],
            "call_us_per_layer": ms_call * 1e3}
        del lay
        torch.cuda.empty_cache()
    return res


# ------------------------------------------------------- N = 1: config 2
def run_single(args, device) -> dict:
    from qwarz_b200 import attention as att
    from qwarz_b200 import build, ops

    build.build()
    stream = torch.cuda.current_stream(device)
    tokens, pages = C2_TOKENS, C2_TOKENS // PAGE
    layers = [build_layer(ops, device, pages, tokens, seed=l) for l in range(LAYERS)]
    q, knew, vnew = new_rows(device, LAYERS)
    out = [torch.empty_like(t) for t in q]
    pre = torch.tensor([tokens - 1], dtype=torch.int32, device=device)
    torch.cuda.synchronize()
    splits = ops.default_splits(device, tokens, 1)
    po, pml = ops.split_workspace(device, 1, splits)

    def step():
        for l in range(LAYERS):
            cache, perm = layers[l]
            ops.nvfp4_attend(q[l], knew[l], vnew[l], *cache, perm, pre, out[l], po, pml, splits)

    def split_only():
        for l in range(LAYERS):
            cache, perm = layers[l]
            ops.attn_split(q[l], cache[0], cache[1], perm, pre, po, pml, cache[2], cache[3], splits)

    graph = capture(step, args.warmup)
    split_graph = capture(split_only, args.warmup)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    with ClockSampler(device.index) as clocks:
        ms_step = cuda_time(graph.replay, args.steps, stream) / args.steps
        torch.cuda.synchronize()
        split_ms_launch = cuda_time(split_graph.replay, args.steps, stream) / args.steps / LAYERS
        torch.cuda.synchronize()
    del graph, split_graph

    # ----- end to end through the drop-in: qwarz_b200.attention.attend per
    # layer (validation, the adapter's persistent output buffer, one append +
    # split + combine), inside the caller's CUDA graph as the engine captures
    # its forward; one pinned H2D of the step's q/k/v, one D2H of the outputs.
    per_in = HEADS * DIM + 2 * KV_HEADS * DIM
    host_in = torch.empty(LAYERS, per_in, dtype=torch.bfloat16).pin_memory()
    for l in range(LAYERS):
        host_in[l].copy_(torch.cat([q[l].flatten(), knew[l].flatten(), vnew[l].flatten()]).cpu())
    host_out = torch.empty(LAYERS, HEADS * DIM, dtype=torch.bfloat16).pin_memory()
    dev_in = torch.empty(LAYERS, per_in, dtype=torch.bfloat16, device=device)
    dq = [dev_in[l, :HEADS * DIM].view(1, 1, HEADS, DIM) for l in range(LAYERS)]
    dk = [dev_in[l, HEADS * DIM:HEADS * DIM + KV_HEADS * DIM].view(1, 1, KV_HEADS, DIM) for l in range(LAYERS)]
    dv = [dev_in[l, HEADS * DIM + KV_HEADS * DIM:].view(1, 1, KV_HEADS, DIM) for l in range(LAYERS)]
    tables = [perm.view(1, -1) for _, perm in layers]
    pre_dev = torch.tensor([tokens - 1], dtype=torch.int32, device=device)

    dev_out = torch.empty(LAYERS, HEADS * DIM, dtype=torch.bfloat16, device=device)

    def e2e_step():
        dev_in.copy_(host_in, non_blocking=True)
        outs = [att.attend(dq[l], dk[l], dv[l], layers[l][0], pre_dev, block_table=tables[l]).view(1, -1)
                for l in range(LAYERS)]
        # the 16 outputs (the adapter's persistent buffers) gathered on the
        # device, then one D2H of the step's result
        torch.cat(outs, dim=0, out=dev_out)
        host_out.copy_(dev_out, non_blocking=True)

    e2e_graph = capture(e2e_step, args.warmup)
    for _ in range(args.warmup):
        e2e_graph.replay()
    torch.cuda.synchronize()
    e2e_ms = cuda_time(e2e_graph.replay, args.steps, stream) / args.steps
    torch.cuda.synchronize()
    del e2e_graph
    # the same calls eagerly (host-bound: Python validation and dispatch)
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    eager_iters = max(3, min(args.steps, 20))
    t0 = time.perf_counter()
    for _ in range(eager_iters):
        e2e_step()
    torch.cuda.synchronize()
    eager_ms = (time.perf_counter() - t0) * 1e3 / eager_iters
    att.release_attention_plans()

    h2d = host_in.numel() * host_in.element_size()
    d2h = host_out.numel() * host_out.element_size()
    bytes_layer = layer_bytes(tokens, 1, pages)
    total_bytes = LAYERS * bytes_layer
    pk, pk_kind = peaks()
    achieved = bytes_layer / (split_ms_launch * 1e-3) / 1e9
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
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": DTYPE,
        "data": DATA,
        "config": {
            "workload": ("C2: decode q_len=1, 16 attention layers x 65,536 tokens NVFP4 KV "
                         "(256 pages of 256, seed-permuted tables), GQA 24/4 x 256"),
            "layers": LAYERS, "context_tokens": tokens, "tokens_per_gpu": tokens,
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
            "algorithmic_bytes_per_launch": bytes_layer,
        },
        "e2e": {
            "value": total_bytes / (e2e_ms * 1e-3) / 1e9,
            "unit": "GB/s",
            "us_per_step": e2e_ms * 1e3,
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": ("qwarz_b200.attention.attend per layer (the drop-in boundary: validation, "
                    "persistent output, append + split + combine), inside the caller's CUDA graph; "
                    "one pinned H2D of the step's q/k/v; the 16 outputs gathered on the device "
                    "(torch.cat) and one D2H"),
            "eager_us_per_step": eager_ms * 1e3,
            "eager_note": "the same 16 attend() calls and copies without a graph (host-bound Python dispatch)",
        },
        # our kernels per timed step: the decode split (append fused) and
        # the combine, per layer
        "gpu_launches": args.steps * LAYERS * 2,
        "clocks": clocks.summary(),
    }
    if not args.no_cpu_baseline:
        sample = [(tuple(t.cpu() for t in layers[i][0]), layers[i][1].cpu(), q[i].view(1, HEADS, DIM).float().cpu())
                  for i in range(2)]
        result["cpu_baseline"] = cpu_oracle_sample(sample, tokens, args.cpu_seconds)
    del layers
    torch.cuda.empty_cache()
    if not args.no_extras:
        extras = {}
        extras["c3_verify"] = c3_record(ops, device, stream, args, pk)
        extras["c4_262144_one_gpu"] = nvfp4_config(ops, device, stream, args, pk, C4_TOKENS, 4)["q1"]
        extras["c5_draft_fp8"] = c5_record(device, stream, args, pk)
        extras["k8v4"] = k8v4_record(device, stream, args, pk)
        extras["prefill"] = prefill_record(ops, device, stream, args, pk)
        result["configs"] = extras
    return result


# ----------------------------------------------- N > 1: config 4 sharded
def run_sharded(args, rank: int, world: int, device) -> dict | None:
    from qwarz_b200 import build, ops, sharded

    build.build()
    dist = torch.distributed
    stream = torch.cuda.current_stream(device)
    total_pages = C4_TOKENS // PAGE
    shard = sharded.shard_pages(total_pages, world)[rank]
    local_pages, local_tokens = shard.num_pages, shard.tok_span
    layers = [build_layer(ops, device, local_pages, local_tokens, seed=l, first_token=shard.tok_begin,
                          perm_seed=100_000 * (rank + 1) + l) for l in range(LAYERS)]
    q, knew, vnew = new_rows(device, LAYERS)
    out = [torch.empty_like(t) for t in q]
    pre = torch.tensor([C4_TOKENS - 1], dtype=torch.int32, device=device)
    torch.cuda.synchronize()
    splits = ops.default_splits(device, local_tokens, 1)
    dec = sharded.ShardedDecode(shard, device, 1, splits, exchange=args.exchange)
    exchange = dec.exchange

    def step():
        for l in range(LAYERS):
            cache, perm = layers[l]
            dec.step(q[l], knew[l], vnew[l], cache, perm, pre, out[l])

    def split_only():  # the shard split kernel alone (append fused on the owner)
        for l in range(LAYERS):
            cache, perm = layers[l]
            ops.shard_split(q[l], knew[l], vnew[l], *cache, perm, pre, dec.partial_o, dec.partial_ml,
                            shard.tok_begin, shard.tok_span, splits)

    def exchange_only():  # merge + exchange + merge of the last partials (a collective)
        for l in range(LAYERS):
            if exchange == "peer":
                ops.shard_exchange_combine(dec.partial_o, dec.partial_ml, splits, dec.peer.peers,
                                           dec.peer.nbytes, dec.peer.epochs, rank, world, out[l])
            else:
                sharded.exchange_records(dec.send, dec.gathered, dec.group)
                ops.combine_gathered(dec.gathered, out[l], world)

    def barrier():
        dist.barrier(device_ids=[device.index])
        torch.cuda.synchronize()

    def timed(graph, collective: bool) -> float:
        for _ in range(args.warmup):
            graph.replay()
        barrier()
        if collective:  # aligns the ranks' start events (see the module doc)
            graph.replay()
        return cuda_time(graph.replay, args.steps, stream) / args.steps

    graph = capture(step, args.warmup)
    split_graph = capture(split_only, args.warmup)
    exch_graph = capture(exchange_only, args.warmup)
    barrier()
    with ClockSampler(device.index) as clocks:
        ms_step = timed(graph, True)
        split_ms = timed(split_graph, False) / LAYERS
        exch_ms = timed(exch_graph, True) / LAYERS
        barrier()
    # leave the outputs of one real step in out[]
    graph.replay()
    torch.cuda.synchronize()
    del graph, split_graph, exch_graph

    # ----- end to end through ShardedDecode.step, host copies in the graph
    per_in = HEADS * DIM + 2 * KV_HEADS * DIM
    host_in = torch.empty(LAYERS, per_in, dtype=torch.bfloat16).pin_memory()
    for l in range(LAYERS):
        host_in[l].copy_(torch.cat([q[l].flatten(), knew[l].flatten(), vnew[l].flatten()]).cpu())
    host_out = torch.empty(LAYERS, HEADS * DIM, dtype=torch.bfloat16).pin_memory()
    dev_in = torch.empty(LAYERS, per_in, dtype=torch.bfloat16, device=device)
    dev_out = torch.empty(LAYERS, HEADS * DIM, dtype=torch.bfloat16, device=device)
    dq = [dev_in[l, :HEADS * DIM].view(1, 1, HEADS, DIM) for l in range(LAYERS)]
    dk = [dev_in[l, HEADS * DIM:HEADS * DIM + KV_HEADS * DIM].view(1, 1, KV_HEADS, DIM) for l in range(LAYERS)]
    dv = [dev_in[l, HEADS * DIM + KV_HEADS * DIM:].view(1, 1, KV_HEADS, DIM) for l in range(LAYERS)]
    do = [dev_out[l].view(1, 1, HEADS, DIM) for l in range(LAYERS)]

    def e2e_step():
        dev_in.copy_(host_in, non_blocking=True)
        for l in range(LAYERS):
            cache, perm = layers[l]
            dec.step(dq[l], dk[l], dv[l], cache, perm, pre, do[l])
        host_out.copy_(dev_out, non_blocking=True)

    e2e_graph = capture(e2e_step, args.warmup)
    e2e_ms = timed(e2e_graph, True)
    barrier()
    del e2e_graph

    # ----- per-rank times; check the outputs across ranks
    times = torch.tensor([ms_step, split_ms, exch_ms, e2e_ms], dtype=torch.float64, device=device)
    all_times = torch.empty(world, 4, dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(all_times, times)
    outs = torch.empty(world, *out[0].shape, dtype=out[0].dtype, device=device)
    dist.all_gather_into_tensor(outs, out[0].contiguous())
    barrier()  # every rank is done with the peer buffers before any rank frees its own
    dec.close()
    del layers
    torch.cuda.empty_cache()

    one_gpu = None
    check = None
    if rank == 0:
        # the same 16-layer step on this GPU alone (rows identical to the
        # shards', one 262,144-token pool per layer), and its layer-0 output
        full = [build_layer(ops, device, total_pages, C4_TOKENS, seed=l, perm_seed=55_555 + l)
                for l in range(LAYERS)]
        s1 = ops.default_splits(device, C4_TOKENS, 1)
        po1, pml1 = ops.split_workspace(device, 1, s1)
        out1 = [torch.empty_like(t) for t in q]

        def step1():
            for l in range(LAYERS):
                cache, perm = full[l]
                ops.nvfp4_attend(q[l], knew[l], vnew[l], *cache, perm, pre, out1[l], po1, pml1, s1)

        ms1 = graph_ms(step1, args.warmup, args.steps, stream)
        step1()
        torch.cuda.synchronize()
        ref = out1[0].float()
        same = all(torch.equal(outs[g], outs[0]) for g in range(world))
        diff = (outs[0].float() - ref).abs()
        excess = float((diff - (2e-3 + ulp_bf16(ref))).max())
        check = {"ranks_bit_identical": same, "layer": 0,
                 "max_abs_vs_one_gpu": float(diff.max()),
                 "tolerance": "2e-3 + 1 BF16 ulp at |one-GPU output| (the parity tests' bound)",
                 "ok": bool(same and excess <= 0)}
        one_gpu = {"us_per_step": ms1 * 1e3, "splits": s1,
                   "note": "the same 16 layers x 262,144 tokens (identical K/V rows) on rank 0's GPU alone, "
                           "one qwz_nvfp4_attend per layer, one CUDA graph"}
        del full
        torch.cuda.empty_cache()
    barrier()
    if rank != 0:
        return None

    t = all_times.cpu()
    ms_step, split_ms, exch_ms, e2e_ms = (float(t[:, i].max()) for i in range(4))
    bytes_local = [layer_bytes(s.tok_span, 1, s.num_pages) for s in sharded.shard_pages(total_pages, world)]
    total_bytes = LAYERS * sum(bytes_local)
    pk, pk_kind = peaks()
    achieved = bytes_local[0] / (split_ms * 1e-3) / 1e9
    return {
        "metric": METRIC,
        "value": total_bytes / (ms_step * 1e-3) / 1e9,
        "unit": "GB/s",
        "us_per_step": ms_step * 1e3,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": DTYPE,
        "data": DATA,
        "config": {
            "workload": (f"C4: decode q_len=1, 16 layers x 262,144 tokens NVFP4 KV (1,024 pages) split "
                         f"contiguously over {world} GPUs ({local_tokens} tokens per GPU); (m,l,O) records "
                         + ("exchanged over NVLink peer memory inside the merge kernel"
                            if exchange == "peer" else "all-gathered by NCCL") + " + LSE combine"),
            "layers": LAYERS, "context_tokens": C4_TOKENS, "tokens_per_gpu": local_tokens,
            "q_len": 1, "heads": "24q/4kv", "head_dim": DIM, "page": PAGE, "splits_per_head": splits,
            "exchange": exchange,
            "l2": f"inputs larger than L2: 16 layers x {bytes_local[0] / 1e6:.1f} MB KV per GPU rotate per step",
            "graph": "one CUDA graph per step",
            "timing": "an untimed replay right before each rank's start event aligns the ranks; "
                      "max over ranks",
        },
        "per_rank_us_per_step": [float(x) * 1e3 for x in t[:, 0]],
        "exchange_us_per_layer": exch_ms * 1e3,
        "one_gpu_same_workload": one_gpu,
        "check": check,
        "roofline": {
            "bound": "hbm",
            "kernel": "nvfp4_decode_kernel via qwz_attn_shard_split (the shard split alone, append fused)",
            "achieved": achieved,
            "peak": pk["hbm_gbs"],
            "peak_kind": pk_kind,
            "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"],
            "traffic": None,
            "us_per_launch": split_ms * 1e3,
            "algorithmic_bytes_per_launch": bytes_local[0],
        },
        "e2e": {
            "value": total_bytes / (e2e_ms * 1e-3) / 1e9,
            "unit": "GB/s",
            "us_per_step": e2e_ms * 1e3,
            "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
            "d2h_bytes_per_step": host_out.numel() * host_out.element_size(),
            "api": f"qwarz_b200.sharded.ShardedDecode.step per layer ({exchange} exchange inside); one "
                   "pinned H2D of the step's q/k/v and one D2H of its outputs per rank; one CUDA graph, "
                   "max over ranks",
        },
        "gpu_launches": args.steps * LAYERS * (2 if exchange == "peer" else 4),
        "clocks": clocks.summary(),
    }


# ------------------------------------------------- other BASELINE configs
def prefill_record(ops, device, stream, args, pk):
    """The prefill kernels: the NVFP4 prefill (one launch over the pages)
    against the 8-row-window route through the verify kernel it replaces,
    and the draft-model prefill (FP16 K/V read in place) against the
    reference's torch SDPA route for the same shapes, each at 8,192 new rows
    onto an empty cache and 4,096 onto 61,440."""
    res = {}
    g = torch.Generator(device=device).manual_seed(7)
    dtype = torch.bfloat16
    # NVFP4 prefill: one launch over the pages vs the 8-row-window route
    # through the verify kernel it replaces
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
        ms_w = graph_ms(windows, 1, 2, stream)  # the old route, graph-captured
        flops = 4 * HEADS * DIM * sum(pre + s + 1 for s in range(S))
        res[f"prefill_{pre}+{S}"] = {
            "pre": pre, "q_len": S, "us_per_layer": ms * 1e3, "TFLOPs": flops / (ms * 1e-3) / 1e12,
            "tensor_frac_of_measured_bf16": flops / (ms * 1e-3) / 1e12 / pk.get("bf16_tflops", 1590.0),
            "windowed_verify_us": ms_w * 1e3, "speedup_vs_windows": ms_w / ms}
        del c, perm
        torch.cuda.empty_cache()
    # draft-model prefill: FP16 K/V read in place vs the reference's torch
    # route for the same shapes (draft.py:33-86: SDPA causal when S == T,
    # else the LSE merge of two flash calls)
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
        res[f"draft_prefill_{pre}+{S}"] = {
            "pre": pre, "q_len": S, "us_per_layer": ms * 1e3, "TFLOPs": flops / (ms * 1e-3) / 1e12,
            "tensor_frac_of_measured_bf16": flops / (ms * 1e-3) / 1e12 / pk.get("bf16_tflops", 1590.0),
            "torch_sdpa_route_us": ms_ref * 1e3, "sdpa_heads_repeated": expand[0],
            "speedup_vs_sdpa_route": ms_ref / ms}
        del qd, kd, vd, outd
        torch.cuda.empty_cache()
    return res


def run_extra(args, device) -> dict:
    """--workload c3|c4|c5|prefill|all: the other configs on one GPU, one
    JSON object (not the driver's headline line)."""
    from qwarz_b200 import build, ops

    build.build()
    stream = torch.cuda.current_stream(device)
    pk, pk_kind = peaks()
    res = {"workload": args.workload, "peak_gbs": pk["hbm_gbs"], "peak_kind": pk_kind, "configs": {}}
    g = torch.Generator(device=device).manual_seed(7)
    dtype = torch.bfloat16
    if args.workload in ("c3", "all"):
        res["configs"]["c3_verify"] = c3_record(ops, device, stream, args, pk)
    if args.workload in ("prefill", "all"):
        res["configs"].update(prefill_record(ops, device, stream, args, pk))
    if args.workload in ("c4", "all"):
        res["configs"]["c4_262144_one_gpu"] = nvfp4_config(ops, device, stream, args, pk, C4_TOKENS, 4)["q1"]
    if args.workload in ("c5", "all"):
        res["configs"]["c5_draft_fp8"] = c5_record(device, stream, args, pk)
    if args.workload in ("k8v4", "all"):
        res["configs"]["k8v4"] = k8v4_record(device, stream, args, pk)
    return res


def run_profile_case(args, device) -> dict:
    """Small case for ncu --set full: one 65,536-token layer (75.5 MB, above
    the L2 working set only with ncu's cache flush between passes), three
    eager launches of the decode split, the q_len 7 verify split, or the FP8
    draft decode."""
    from qwarz_b200 import build, ops
    from qwarz_b200.draft_attention import DecodeAttention

    build.build()
    tokens, pages = C2_TOKENS, C2_TOKENS // PAGE
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
    if args.workload == "profile_k8v4":
        from qwarz_b200 import k8v4

        cache, perm = k8v4_layer(device, pages, tokens, 9000)
        q = torch.randn(1, HEADS, DIM, generator=g, device=device).bfloat16()
        pre = torch.tensor([tokens - 1], dtype=torch.int32, device=device)
        splits = ops.default_splits(device, tokens, 1)
        po, pml = ops.split_workspace(device, 1, splits)
        out = torch.empty_like(q)
        h32 = k8v4.hadamard32(device)
        for _ in range(3):
            k8v4.split(q, cache, perm, pre, po, pml, h32, splits)
            k8v4.combine(po, pml, out, h32, splits)
        torch.cuda.synchronize()
        return {"workload": args.workload, "tokens": tokens, "ok": True}
    if args.workload in ("profile_draft", "profile_draft16"):
        T = tokens + 6
        k8 = torch.randn(1, T, KV_HEADS, DIM, generator=g, device=device).to(torch.float8_e4m3fn)
        v8 = torch.randn(1, T, KV_HEADS, DIM, generator=g, device=device).to(torch.float8_e4m3fn)
        q = torch.randn(1, 1, HEADS, DIM, generator=g, device=device).half()
        out = torch.empty_like(q)
        # profile_draft16: BASELINE's 16 chunks (each chunk a cluster of CTAs)
        attn = DecodeAttention(HEADS, KV_HEADS, DIM, device, **({"splits": 16} if args.workload.endswith("16") else {}))
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
def run_reference(args, world: int) -> dict:
    """The reference's CPU oracle path, restated (oracle/), on host cores:
    NVFP4 -> dequant gather (xqa.py:73-143) + FP32 softmax attention
    (xqa.py:612-673).  One step is one layer call of the arm's workload: a
    65,536-token layer (config 2) at N = 1, the whole 262,144-token layer
    (config 4; the CPU path is not sharded) at N > 1."""
    import numpy as np
    from oracle import attention as oatt
    from oracle import nvfp4

    torch.set_num_threads(os.cpu_count() or 1)
    tokens = C2_TOKENS if world == 1 else C4_TOKENS
    pages = tokens // PAGE
    layers = []
    for l in range(2 if world == 1 else 1):
        g = torch.Generator().manual_seed(900 + l)
        outl = torch.randperm(DIM, generator=g)[:4]
        k = torch.randn(tokens, KV_HEADS, DIM, generator=g)
        v = torch.randn(tokens, KV_HEADS, DIM, generator=g)
        k[..., outl] *= 8
        v[..., outl] *= 8
        k, v = k.numpy(), v.numpy()
        kc, ks = nvfp4.quantize_rows(k)
        vc, vs = nvfp4.quantize_rows(v)
        del k, v
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
    workload = ("C2 sample: one 65,536-token q_len=1 decode layer call per step" if world == 1 else
                "C4 sample: one 262,144-token q_len=1 decode layer call per step (the whole sequence "
                "on rank 0's host cores; the CPU path is not sharded)")
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "us_per_step": per * 1e6,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "NVFP4 KV dequantised to FP32; FP32 softmax attention",
        "data": "synthetic (seeded N(0,1) K/V with 4 outlier channels x8, NVFP4 by the oracle writer)",
        "config": {"workload": workload, "step": "one layer call", "context_tokens": tokens},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{args.steps} layer calls after {args.warmup} warm-up, "
                                   f"{per * 1e3:.1f} ms per layer call"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="N=1: leave out the config 3/4/5 sub-records")
    ap.add_argument("--exchange", default="auto", choices=["auto", "peer", "nccl"],
                    help="N>1: exchange of the shard records (auto: NVLink peer memory when every "
                         "rank can reach every GPU, else NCCL)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--workload", default="auto",
                    choices=["auto", "c3", "c4", "c5", "k8v4", "prefill", "all", "profile_prefill",
                             "profile_decode", "profile_verify", "profile_draft", "profile_draft16",
                             "profile_k8v4"],
                    help="auto: the driver's headline (config 2 at N=1 with sub-records, config 4 "
                         "split over the N GPUs at N>1); c3/c4/c5/k8v4/prefill/all: single-GPU configs "
                         "(separate JSON); profile_*: three eager launches of one kernel on one "
                         "65,536-token layer, the small case for ncu --set full")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(run_reference(args, world)), flush=True)
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.workload.startswith("profile_"):
        print(json.dumps(run_profile_case(args, device)), flush=True)
        return
    if args.workload != "auto":
        print(json.dumps(run_extra(args, device)), flush=True)
        return
    if world == 1:
        result = run_single(args, device)
    else:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
        try:
            result = run_sharded(args, rank, world, device)
        finally:
            torch.distributed.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
