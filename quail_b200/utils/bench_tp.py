"""Tensor-parallel benchmark: AI.IF prefill on Qwen3-32B fp8 (random init), TP = N GPUs.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m quail_b200.utils.bench_tp \
        [--steps K] [--warmup W] [--comm fused|nccl] [--chunk-tokens 32768]

All ranks run the same packed chunks (rows lognormal(median 400, sigma 0.6)
clipped to [16, 4096], a 48-token shared prefix); one step is one forward
pass. --query if_classify adds AI.CLASSIFY (4 labels) on the rows AI.IF keeps:
its questions read the document's pages and need full-vocabulary readouts,
so the timed passes mix new documents with classify follow-ups. Device-timed with CUDA events over exactly K steps, max over ranks.
--comm fused: the in-kernel AG->GEMM / GEMM->RS paths; --comm nccl: the
same GEMMs with NCCL all-gather / reduce-scatter between them (baseline).
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
    ap.add_argument("--model", default="qwen3-32b-fp8")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--chunk-tokens", type=int, default=32768)
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--query", default="if", choices=["if", "if_classify"],
                    help="if: AI.IF alone; if_classify: AI.IF, then AI.CLASSIFY into 4 labels (1-3 seeded token "
                         "ids each) on the rows it keeps (BASELINE config 4)")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    rank, world = dist.get_rank(), dist.get_world_size()
    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.parallel.tp import TPQwen3
    from quail_b200.utils.synthetic import make_workload, rows_for_tokens

    cfg = MODEL_CONFIGS[args.model]
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    rng = np.random.default_rng(11)
    labels = [[int(x) for x in rng.integers(1000, 100000, int(rng.integers(1, 4)))] for _ in range(4)]
    answer = list(range(8))
    for lab in labels:
        for t in lab:
            if t not in answer:
                answer.append(t)
    model = TPQwen3(cfg, dist.group.WORLD, seed=0, max_tokens=args.chunk_tokens + 4096, answer_ids=answer,
                    comm=args.comm)
    pages = 2 * (args.chunk_tokens // 128) + 512
    arena = KVArena(cfg.layers, pages, 128, cfg.num_kv_heads // world, 128, device=dev)
    steps = args.warmup + args.steps + 2
    wl = make_workload(rows_for_tokens(steps * args.chunk_tokens * 1.1, median=400), median=400, sigma=0.6,
                       hi=4096, seed=7)  # the same rows on every rank
    ex = StageExecutor(model, arena, args.chunk_tokens)
    call = Call(kind="filter", suffix=wl.suffix, true_cols=[0, 1, 2, 3], false_cols=[4, 5, 6, 7], name="if")
    calls = [call]
    if args.query == "if_classify":
        suffix2 = np.random.default_rng(12).integers(0, cfg.vocab, 56).astype(np.int32)
        calls.append(Call(kind="classify", suffix=suffix2, name="kind", labels=[np.asarray(x, np.int32) for x in labels],
                          label_cols=[[answer.index(t) for t in lab] for lab in labels]))
    run = RegionRun(ex, wl.prefix, wl.bodies, calls, answer_width=len(answer))
    run.submit_all()
    ex.step()
    for _ in range(args.warmup):
        ex.step()
    torch.cuda.synchronize()
    dist.barrier()
    tok0, passes0 = ex.stats.tokens, ex.stats.passes
    model.timer.reset()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        ex.step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    fresh = ex.stats.tokens - tok0
    rows = sum(ex.stats.pass_rows[passes0:])
    ops_ms = model.timer.summary()  # QB_OP_TIMING=1: device ms per op over the timed steps (this rank)
    err = model.check_errors()
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t[0])
    if rank == 0:
        prompt = fresh + rows * len(wl.prefix)
        print(json.dumps({"metric": f"AI.{'IF + AI.CLASSIFY' if args.query == 'if_classify' else 'IF'} prefill "
                                    f"tok/s, qwen3-32b-fp8 tensor-parallel", "comm": args.comm, "query": args.query,
                          "tp": world, "layers": cfg.layers, "value": round(prompt / (ms_max / 1e3), 1),
                          "unit": "prompt tokens/s", "rows_per_second": round(rows / (ms_max / 1e3), 1),
                          "fresh_tokens_per_second": round(fresh / (ms_max / 1e3), 1),
                          "ms_per_step": round(ms_max / args.steps, 3), "steps": args.steps,
                          "chunk_tokens": args.chunk_tokens, "kernel_error": err,
                          **({"op_ms_rank0": ops_ms} if ops_ms else {})}), flush=True)
    dist.barrier()
    del model
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
