"""Run by tests/test_gpu_multi.py under torch.distributed.run, one process
per GPU: the sequence-sharded decode (ShardedDecode) with the peer-memory
exchange and with NCCL, eager and replayed from a CUDA graph, against the
FP32 oracle over the whole sequence; then the MTP7 verify over the peer
exchange with its 7 new rows across the shard boundary at token 2048 (the
owners write them inside their verify kernels).  Prints one JSON line per
rank and exits non-zero on a mismatch."""
from __future__ import annotations

import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from oracle import attention as oatt  # noqa: E402
from oracle import nvfp4, rng  # noqa: E402
from qwarz_b200 import _lib, sharded  # noqa: E402
from tests.conftest import assert_close_attention  # noqa: E402
from tests.golden import cases  # noqa: E402
from tests.gpu_helpers import make_cache, queries, to_cpu_torch, to_device  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    device = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=device)
    total, pages = 3000, 16
    table = rng.permutation(77, pages)
    c, _, _ = make_cache(780, total, pages, table)
    ref = {n: c[n].copy() for n in ("k_cache", "v_cache", "k_scales", "v_scales", "table")}
    shard = sharded.shard_pages(pages, world)[rank]
    phys = table[shard.first_page:shard.first_page + shard.num_pages]
    results = {}
    for mode, q_len in (("peer", 1), ("nccl", 1), ("peer", 7)):
        d = {n: np.ascontiguousarray(c[n][phys]) for n in ("k_cache", "v_cache", "k_scales", "v_scales")}
        d["table"] = np.arange(shard.num_pages, dtype=np.int32)
        dc = to_device(d, device)
        cache = (dc["k_cache"], dc["v_cache"], dc["k_scales"], dc["v_scales"])
        dec = sharded.ShardedDecode(shard, device, q_len=q_len, exchange=mode)
        refm = {n: v.copy() for n, v in ref.items()}
        q = queries(31 if q_len == 1 else 41, q_len, torch.bfloat16).to(device)
        out = torch.empty_like(q)
        errs = []
        lens = torch.zeros(1, dtype=torch.int32, device=device)
        kd = torch.empty(q_len, 4, 256, dtype=torch.bfloat16, device=device)
        vd = torch.empty_like(kd)
        graph = None
        start = total if q_len == 1 else 2045  # verify: rows 2045.. cross the page-8 shard boundary
        for step in range(4):  # steps 0-1 eager, 2-3 replayed from one CUDA graph
            pre = start + step
            kn = torch.from_numpy(cases.kv_rows(600 + step, q_len)).to(torch.bfloat16)
            vn = torch.from_numpy(cases.kv_rows(700 + step, q_len)).to(torch.bfloat16)
            nvfp4.append(kn.float().numpy(), vn.float().numpy(), refm["k_cache"], refm["v_cache"],
                         refm["k_scales"], refm["v_scales"], table, pre)
            lens.fill_(pre)
            kd.copy_(kn)
            vd.copy_(vn)
            if step < 2:
                dec.step(q, kd, vd, cache, dc["table"], lens, out)
            else:
                if graph is None:
                    torch.cuda.synchronize()
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph):
                        dec.step(q, kd, vd, cache, dc["table"], lens, out)
                graph.replay()
            torch.cuda.synchronize()
            expect = oatt.nvfp4_attention(q.float().cpu(), **{k: v for k, v in to_cpu_torch(refm).items()
                                                               if k != "table"},
                                          block_table=torch.from_numpy(table), pre_len=pre)
            try:
                assert_close_attention(out.float().cpu().numpy(), expect.numpy(), f"{mode} q_len {q_len} step {step}",
                                       "bfloat16")
            except AssertionError as e:
                errs.append(str(e))
            if graph is not None and step == 2:
                # the capture ran the step once more on the same position: undo nothing, the
                # append is idempotent for the same row and the same position
                pass
        del graph
        errs += [] if _lib.device_error(clear=True) == 0 else ["device error word set"]
        results[f"{mode}_q{q_len}"] = errs or "ok"
        dec.close()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    print(json.dumps({"rank": rank, "world": world, "results": results}))
    return 0 if all(v == "ok" for v in results.values()) else 1


if __name__ == "__main__":
    sys.exit(main())
