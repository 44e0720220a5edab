"""Flagship benchmark: AI.IF over synthetic rows on Qwen3-4B fp8 (random init).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step is one packed prefill pass of `--chunk-tokens` (16,384) new tokens:
many rows' documents + question, each reading the shared 48-token template
prefix through the paged arena, with the yes/no readout of every finished
row. Rows are sharded data-parallel: every rank runs its own rows (weak
scaling; with N > 1 launch with torchrun, one rank per GPU over NCCL).

value: prompt tokens per second over all ranks (every prompt's full length
with the shared prefix counted each time, the reference's
input_tokens_per_second), device-timed with CUDA events over exactly K
steps, max over ranks. rows/s and fresh (computed) tokens/s are reported
beside it. e2e: the same run through the session API (SQL AI.IF query over a
registered table) with its host->device inputs and device->host answers
inside the timed region.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_TOKS_PER_GPU = 17_000.0   # H100 SXM, qwen3-4b-fp8 prompt tok/s per GPU (the published reference number)
METRIC = "AI-function rows/sec & prefill tok/s per box (AI.IF, qwen3-4b-fp8), device-timed"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="qwen3-4b-fp8")
    ap.add_argument("--chunk-tokens", type=int, default=16384)
    ap.add_argument("--pages", type=int, default=1024)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-rows", type=int, default=200_000,
                    help="rows of the end-to-end query's table over all ranks (the configuration's 200k)")
    ap.add_argument("--profile-pass", action="store_true",
                    help="after the timed steps, run one more pass between cudaProfilerStart/Stop "
                         "(for `ncu --profile-from-start off`); it is not timed")
    return ap.parse_args()


def reference_arm(args):
    line = {"impl": "reference", "metric": METRIC, "n_gpus": args.gpus,
            "unavailable": ("the reference cannot be installed offline: its build backend is maturin "
                            "(Rust extension _quail_native) and neither maturin nor a Rust toolchain is in "
                            "this image; it also pins vllm==0.29.0 (0.22 installed)")}
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)

    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor
    from quail_b200.models.build import SYNTHETIC_FALSE_IDS, SYNTHETIC_TRUE_IDS, build_pipeline
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.utils.clocks import ClockSampler
    from quail_b200.utils.synthetic import make_workload, rows_for_tokens

    cfg = MODEL_CONFIGS[args.model]
    pipe = build_pipeline(cfg, device=dev, seed=0, max_tokens=args.chunk_tokens + 256)
    from quail_b200.planner.budgets import Budgets
    slots = Budgets.for_model(cfg, "b200", gpus=1).state_slots(cfg) if cfg.is_hybrid else 0
    arena = KVArena.for_model(cfg, args.pages, 128, device=dev, state_slots=slots)
    nt = len(SYNTHETIC_TRUE_IDS)

    def call(suffix):
        if cfg.canvas_tokens:
            # a canvas model (DiffusionGemma) reads its answer at the canvas row after the question
            from quail_b200.models.gemma4 import canvas_ids
            suffix = np.concatenate([suffix, canvas_ids(cfg)]).astype(np.int32)
        return Call(kind="filter", suffix=suffix, true_cols=list(range(nt)), false_cols=list(range(nt, 2 * nt)),
                    name="if")

    # ---------------------------------------------------------------- device-timed steps
    steps_total = args.warmup + args.steps + 2
    wl = make_workload(rows_for_tokens(steps_total * args.chunk_tokens * 1.1), seed=1000 + rank)
    ex = StageExecutor(pipe, arena, args.chunk_tokens, gpu_timing=True)
    run = RegionRun(ex, wl.prefix, wl.bodies, [call(wl.suffix)])
    run.submit_all()
    ex.step()  # the shared prefix pass
    for _ in range(args.warmup):
        ex.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local).start()
    tok0, passes0 = ex.stats.tokens, ex.stats.passes
    gpu0 = ex.stats.gpu_ms
    launches0 = ops.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # readouts of the last warm-up pass are collected inside the first timed step
    start.record()
    for _ in range(args.steps):
        if not ex.step():
            raise RuntimeError("workload ran out of rows before the timed steps ended")
    end.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    # device time inside the passes' forward calls (event pairs around each pass): the rest of
    # the timed region is the GPU waiting for the host
    busy_ms = ex.stats.gpu_ms - gpu0
    launches = ops.launch_count() - launches0
    fresh = ex.stats.tokens - tok0
    # rows whose last token ran in the timed passes
    rows_done = sum(ex.stats.pass_rows[passes0:])
    err = ops.read_and_clear_error(local)
    if err:
        raise RuntimeError(f"kernel error code {err}")
    if args.profile_pass:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        ex.step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    # drain the rest of this workload (not timed) so the arena is clean
    while ex.step():
        pass

    import torch as _t
    t = _t.tensor([ms, float(fresh), float(rows_done)], dtype=_t.float64, device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        ms_max = float(mx[0])
    else:
        ms_max = float(t[0])
    fresh_all, rows_all = float(t[1]), float(t[2])
    # each finished row also read the 48 shared tokens: prompt tokens = fresh + rows * prefix
    prompt_all = fresh_all + rows_all * len(wl.prefix)
    toks_per_s = prompt_all / (ms_max / 1e3)

    # ---------------------------------------------------------------- end to end through the API
    e2e = None
    if not args.no_e2e:
        from quail_b200.utils.e2e import run_e2e
        e2e = run_e2e(pipe, arena, cfg, args, rank, world, dev)

    if rank == 0:
        line = {
            "metric": METRIC if args.model == "qwen3-4b-fp8" else METRIC.replace("qwen3-4b-fp8", args.model),
            "value": round(toks_per_s, 1),
            "unit": "prompt tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(toks_per_s / (BASELINE_TOKS_PER_GPU * world), 3),
            "baseline_value": BASELINE_TOKS_PER_GPU * world,
            "rows_per_second": round(rows_all / (ms_max / 1e3), 1),
            "fresh_tokens_per_second": round(fresh_all / (ms_max / 1e3), 1),
            "dtype": ("fp8 e4m3 weights+activations, MX block scaling on the tensor cores: UE8M0 (power-of-two) "
                      "scales per 1x32 activation group and per 128x128 weight block (checkpoint fp32 "
                      "128x128 weight_scale_inv requantized to UE8M0 at load); bf16 KV cache and residual"
                      if cfg.fp8 else "bf16"),
            "data": "synthetic: random token-id bodies lognormal(median 180, sigma 0.6) clipped [16, 2048], "
                    "48-token shared template prefix, 40-token question suffix; random-init weights N(0, 0.02)",
            "config": {"model": ("qwen3-4b-fp8 (36 layers, hidden 2560, 32q/8kv heads, d128, SwiGLU 9728, "
                                 "vocab 151936)" if args.model == "qwen3-4b-fp8" else args.model),
                       "global_batch": f"{args.chunk_tokens} tokens per rank per step",
                       "seq_len": "per row: 48 + body + 40", "parallelism": f"dp{world}",
                       "workload": "AI.IF filter, packed prefill chunks, yes/no readout",
                       "l2": "inputs larger than L2 (4.4 GB of weights streamed every step)"},
            "gpu_launches": launches,
            "forward_ms_per_step": round(busy_ms / args.steps, 3),
            "clocks": clocks,
        }
        if e2e is not None:
            line["e2e"] = e2e
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
