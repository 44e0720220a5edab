"""AI.MAP benchmark on one GPU: greedy decode through the dense kernel pipeline.

    python -m quail_b200.utils.bench_map [--model qwen3-4b-fp8] [--rows 1024] [--max-new 64] [--graphs on|off|both]

Rows are synthetic documents (lognormal lengths, median 250 tokens, a shared
48-token template prefix, a 24-token instruction), prefilled and then
decoded greedily for up to `--max-new` tokens; the stop token never comes
up on random weights, so every row generates `--max-new` tokens. Decode
steps of running rows and prefills of new rows share packed passes; once
every row is admitted, passes are pure decode steps, which run as CUDA graph
replays with `--graphs on` (engine/graphs.py).

Timed: the whole region after a warm-up region (graphs captured there), with
CUDA events on the stream (host gaps included). Prints one JSON line per
graphs setting: rows/s, generated tokens/s, passes, launches.
"""

from __future__ import annotations

import argparse
import json

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-4b-fp8")
    ap.add_argument("--rows", type=int, default=1024)
    ap.add_argument("--warmup-rows", type=int, default=256)
    ap.add_argument("--max-new", type=int, default=64)
    ap.add_argument("--chunk-tokens", type=int, default=16384)
    ap.add_argument("--pages", type=int, default=3072)
    ap.add_argument("--graphs", default="both", choices=["on", "off", "both"])
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)

    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor
    from quail_b200.models.build import build_pipeline
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.utils.clocks import ClockSampler
    from quail_b200.utils.synthetic import make_workload

    cfg = MODEL_CONFIGS[args.model]
    pipe = build_pipeline(cfg, dev, answer_ids=list(range(8)))
    from quail_b200.planner.budgets import Budgets
    # hybrids keep a recurrent state slot per running row beside the KV pages
    slots = Budgets.for_model(cfg, "b200", gpus=1).state_slots(cfg) if cfg.is_hybrid else 0
    arena = KVArena.for_model(cfg, args.pages, 128, device=dev, state_slots=slots)

    def region(rows, seed, graphs):
        wl = make_workload(rows, median=250, sigma=0.6, hi=4096, suffix_tokens=24, seed=seed)
        ex = StageExecutor(pipe, arena, args.chunk_tokens)
        if graphs:
            ex.enable_graphs()
        call = Call(kind="map", suffix=wl.suffix, max_tokens=args.max_new, stop_ids=(151645,), name="map")
        run = RegionRun(ex, wl.prefix, wl.bodies, [call], answer_width=8)
        return wl, ex, run

    modes = {"on": [True], "off": [False], "both": [False, True]}[args.graphs]
    for graphs in modes:
        _, ex0, run0 = region(args.warmup_rows, 5000, graphs)
        g0 = ex0.graphs
        run0.run()
        torch.cuda.synchronize()
        wl, ex, run = region(args.rows, 1000, graphs)
        if graphs:
            ex.graphs = g0          # the warm-up region's captured buckets
        rep0 = g0.replays if graphs else 0
        sampler = ClockSampler(0).start()
        launches0 = ops.launch_count()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        run.run()
        e.record()
        torch.cuda.synchronize()
        clocks = sampler.stop()
        ms = s.elapsed_time(e)
        err = ops.read_and_clear_error(0)
        gen = sum(len(r.values.get("map", [])) for r in run.results)
        sec = ms / 1e3
        print(json.dumps({
            "metric": f"AI.MAP rows/s (greedy decode), {args.model}, 1 GPU, device-timed",
            "graphs": graphs, "value": round(args.rows / sec, 2), "unit": "rows/s",
            "prompt_tokens_per_second": round(wl.prompt_tokens() / sec, 1),
            "generated_tokens_per_second": round(gen / sec, 1), "generated_tokens": gen,
            "passes": ex.stats.passes, "replays": g0.replays - rep0 if graphs else 0,
            "captures": g0.captures if graphs else 0, "seconds": round(sec, 3), "max_new": args.max_new,
            "gpu_launches": ops.launch_count() - launches0, "kernel_error": err, "clocks": clocks,
        }), flush=True)
        del ex, run, ex0, run0


if __name__ == "__main__":
    main()
