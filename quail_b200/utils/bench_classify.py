"""Config-3 benchmark: AI.IF-guarded AI.CLASSIFY + AI.SCORE on Qwen3-8B bf16 (random init), one GPU.

    python -m quail_b200.utils.bench_classify [--steps K] [--warmup W] [--e2e-rows R]

The query reads each row once: AI.IF first; on the rows it keeps, AI.CLASSIFY
into 4 labels (each a seeded 1-3 token id sequence) and AI.SCORE, asked as
follow-up questions over the row's document pages:

    SELECT id, AI.CLASSIFY(body, [4 labels]) AS k, AI.SCORE(PROMPT('...{0}', body)) AS s
    FROM docs WHERE AI.IF(PROMPT('...{0}', body))

Rows: lognormal(median 300, sigma 0.7) bodies clipped to [16, 4096] (100k in
the configuration). Device-timed: exactly K packed passes after W warm-up
passes, CUDA events on the stream; a pass mixes new documents with the
follow-up questions of earlier ones, so rows/s counts rows whose chain
finished inside the timed passes. e2e: the same query through
Session.sql(...).run() over a registered table of `--e2e-rows` rows.
"""

from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b-bf16")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--chunk-tokens", type=int, default=16384)
    ap.add_argument("--pages", type=int, default=2048)
    ap.add_argument("--e2e-rows", type=int, default=5000)
    args = ap.parse_args()
    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor
    from quail_b200.models.build import build_pipeline
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.utils.clocks import ClockSampler
    from quail_b200.utils.synthetic import make_workload, rows_for_tokens

    dev = torch.device("cuda", 0)
    cfg = MODEL_CONFIGS[args.model]
    rng = np.random.default_rng(11)
    labels = [rng.integers(1000, 100000, int(rng.integers(1, 4))).astype(np.int32) for _ in range(4)]
    answer = list(range(8))
    for lab in labels:
        for t in lab:
            if int(t) not in answer:
                answer.append(int(t))
    pipe = build_pipeline(cfg, device=dev, seed=0, answer_ids=answer, max_tokens=args.chunk_tokens + 256)
    arena = KVArena(cfg.layers, args.pages, 128, cfg.num_kv_heads, cfg.head_dim, device=dev)
    steps = args.warmup + args.steps + 2
    wl = make_workload(rows_for_tokens(steps * args.chunk_tokens * 1.2, median=300, sigma=0.7), median=300,
                       sigma=0.7, hi=4096, seed=3)
    fixed = np.random.default_rng(77)
    classify_suffix = fixed.integers(0, 151643, 56).astype(np.int32)
    score_suffix = fixed.integers(0, 151643, 30).astype(np.int32)
    calls = [Call(kind="filter", suffix=wl.suffix, true_cols=[0, 1, 2, 3], false_cols=[4, 5, 6, 7], name="if"),
             Call(kind="classify", suffix=classify_suffix, name="k", labels=labels,
                  label_cols=[[answer.index(int(t)) for t in lab] for lab in labels]),
             Call(kind="score", suffix=score_suffix, true_cols=[0, 1, 2, 3], false_cols=[4, 5, 6, 7], name="s")]
    ex = StageExecutor(pipe, arena, args.chunk_tokens, gpu_timing=True)
    run = RegionRun(ex, wl.prefix, wl.bodies, calls, answer_width=len(answer))
    done = [0]
    run.on_finish = lambda r: done.__setitem__(0, done[0] + 1)
    run.submit_all()
    ex.step()
    for _ in range(args.warmup):
        ex.step()
    torch.cuda.synchronize()
    sampler = ClockSampler(0).start()
    tok0, done0, asked0 = ex.stats.tokens, done[0], run.asked
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        if not ex.step():
            raise RuntimeError("the workload ran out of rows before the timed steps ended")
    e.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = s.elapsed_time(e)
    rows = done[0] - done0
    fresh = ex.stats.tokens - tok0
    asked = run.asked - asked0
    assert ops.read_and_clear_error(0) == 0
    while ex.step():
        pass
    kept = sum(1 for r in run.results if r.values.get("if"))
    line = {"metric": "AI.IF-guarded AI.CLASSIFY + AI.SCORE rows/s (qwen3-8b-bf16), device-timed",
            "value": round(rows / (ms / 1e3), 1), "unit": "rows/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "fresh_tokens_per_second": round(fresh / (ms / 1e3), 1), "questions_per_second":
            round(asked / (ms / 1e3), 1), "pass_rate": round(kept / max(len(run.results), 1), 3),
            "dtype": "bf16", "data": "synthetic: lognormal(median 300, sigma 0.7) token-id bodies clipped "
            "[16, 4096]; random-init weights", "clocks": clocks}
    line["e2e"] = _e2e(pipe, arena, cfg, args, labels)
    print(json.dumps(line), flush=True)


def _e2e(pipe, arena, cfg, args, labels) -> dict:
    import pyarrow as pa

    import quail_b200 as quail
    from quail_b200.api.engine import ModelEngine
    from quail_b200.utils.synthetic import make_workload
    wl = make_workload(args.e2e_rows, median=300, sigma=0.7, hi=4096, seed=9)
    lens = np.array([len(b) for b in wl.bodies])
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    table = pa.table({"id": np.arange(wl.rows), "body": pa.ListArray.from_arrays(
        pa.array(offs), pa.array(np.concatenate(wl.bodies), pa.int32()))})
    config = quail.EngineConfig(model=args.model, device="b200", chunk_tokens=args.chunk_tokens, tokenizer="words")
    s = quail.Session(config=config)
    s.attach_engine(ModelEngine.from_replica(config, pipe, arena))
    s.register("docs", table)
    names = ", ".join(f"'label {i}'" for i in range(4))
    q = s.sql(f"SELECT id, AI.CLASSIFY(body, [{names}]) AS k, "
              f"AI.SCORE(PROMPT('Is the customer satisfied? {{0}}', body)) AS s FROM docs "
              f"WHERE AI.IF(PROMPT('Is this a complaint about a delivery? {{0}}', body))")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    res = q.run()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    return {"value": round(wl.rows / wall, 1), "unit": "rows/s", "rows": wl.rows, "kept_rows": res.table.num_rows,
            "wall_s": round(wall, 3), "asked": res.report.get("asked"),
            "api": "quail_b200.Session.sql(AI.IF-guarded AI.CLASSIFY + AI.SCORE).run()"}


if __name__ == "__main__":
    main()
