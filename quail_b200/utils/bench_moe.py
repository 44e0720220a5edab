"""MoE benchmark: AI.MAP with greedy decode on Qwen3-30B-A3B fp8 (random init), expert-parallel.

    python -m quail_b200.utils.bench_moe [--rows R] [--max-new 64]                 # one GPU, all experts
    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m quail_b200.utils.bench_moe [--comm fused|nccl]

Every rank owns E / N experts and its own rows (R per rank, bodies
lognormal(median 250, sigma 0.6) clipped to [16, 4096], a shared 48-token
template prefix, a 24-token question); each row is prefilled, then decoded
greedily for up to `--max-new` tokens, with the KV arena in 16-token pages.
Rows are admitted continuously: decode steps of running rows and prefills of
new rows share packed passes. Ranks run in lockstep (one pass each per
round; idle ranks still serve their experts).

Timed: the whole region (prefill + decode) after a warm-up region, with CUDA
events on the stream (host gaps included), max over ranks. Reports rows/s
over all ranks, prompt tokens/s and generated tokens/s.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-30b-a3b-fp8")
    ap.add_argument("--rows", type=int, default=1024, help="rows per rank in the timed region")
    ap.add_argument("--warmup-rows", type=int, default=64)
    ap.add_argument("--max-new", type=int, default=64)
    ap.add_argument("--chunk-tokens", type=int, default=16384)
    ap.add_argument("--page-tokens", type=int, default=16)
    ap.add_argument("--kv-gb", type=float, default=60.0)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = cpu_group = None
    rank = 0
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
        rank = dist.get_rank()
        group = dist.group.WORLD
        cpu_group = dist.new_group(backend="gloo", timeout=timedelta(seconds=300))

    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.models.qwen3_moe import Qwen3MoePipeline, Qwen3MoeWeights
    from quail_b200.parallel.ep import run_lockstep
    from quail_b200.utils.clocks import ClockSampler
    from quail_b200.utils.synthetic import make_workload

    cfg = MODEL_CONFIGS[args.model]
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    E = cfg.num_experts
    lo, hi = rank * E // world, (rank + 1) * E // world
    weights = Qwen3MoeWeights(cfg, None, dev, experts=range(lo, hi), head_rows=range(8), seed=0)
    pipe = Qwen3MoePipeline(cfg, weights, max_tokens=args.chunk_tokens + 256, group=group)
    if args.comm == "nccl":
        pipe.ep.comm = "nccl"
    torch.cuda.empty_cache()
    kv_token_bytes = cfg.layers * 2 * cfg.num_kv_heads * cfg.head_dim * 2
    pages = int(args.kv_gb * 1e9 / (kv_token_bytes * args.page_tokens))
    arena = KVArena(cfg.layers, pages, args.page_tokens, cfg.num_kv_heads, cfg.head_dim, device=dev)

    def region(rows, seed):
        wl = make_workload(rows, median=250, sigma=0.6, hi=4096, suffix_tokens=24, seed=seed)
        ex = StageExecutor(pipe, arena, args.chunk_tokens)
        call = Call(kind="map", suffix=wl.suffix, max_tokens=args.max_new, stop_ids=(151645,), name="map")
        run = RegionRun(ex, wl.prefix, wl.bodies, [call], answer_width=8)
        run.submit_all()
        return wl, ex, run

    def drive(ex, run):
        if world > 1:
            run_lockstep(ex, pipe, cpu_group)
        else:
            ex.run()
        ex.free(("prefix",))

    # warm-up region (untimed): compiles nothing, but touches every kernel and buffer
    _, ex0, run0 = region(args.warmup_rows, 5000 + rank)
    drive(ex0, run0)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wl, ex, run = region(args.rows, 1000 + rank)
    pipe.ep.timer.reset()
    sampler = ClockSampler(local).start()
    launches0 = ops.launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    drive(ex, run)
    e.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = s.elapsed_time(e)
    ops_ms = pipe.ep.timer.summary()   # QB_OP_TIMING=1: device ms per MoE step over the timed region (this rank)
    launches = ops.launch_count() - launches0
    err = ops.read_and_clear_error(local)
    gen = sum(len(r.values.get("map", [])) for r in run.results)
    prompt = wl.prompt_tokens()
    t = torch.tensor([ms, float(args.rows), float(prompt), float(gen), float(ex.stats.passes), float(err)],
                     dtype=torch.float64, device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        ms_max, err_max = float(mx[0]), int(mx[5])
    else:
        ms_max, err_max = float(t[0]), int(t[5])
    sec = ms_max / 1e3
    if rank == 0:
        print(json.dumps({
            "metric": "AI.MAP rows/s (greedy decode), qwen3-30b-a3b-fp8 expert-parallel, device-timed",
            "value": round(float(t[1]) / sec, 2), "unit": "rows/s", "n_gpus": world, "comm": args.comm,
            "ep": world, "experts_per_gpu": E // world, "layers": cfg.layers,
            "prompt_tokens_per_second": round(float(t[2]) / sec, 1),
            "generated_tokens_per_second": round(float(t[3]) / sec, 1),
            "rows": int(t[1]), "generated_tokens": int(t[3]), "passes_max": int(mx[4]) if world > 1 else int(t[4]),
            "seconds": round(sec, 3), "max_new": args.max_new, "page_tokens": args.page_tokens,
            "chunk_tokens": args.chunk_tokens, "gpu_launches": launches, "kernel_error": err_max,
            **({"op_ms_rank0": ops_ms} if ops_ms else {}),
            "clocks": clocks,
        }), flush=True)
    if world > 1:
        dist.barrier()
        del pipe
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
