"""End-to-end timing of the flagship query through the public API.

The timed region covers what a user's call pays per step: packing each
chunk on the host, its host->device copy from pinned memory, the forward
pass, and the device->host read of the answers, wall-clock with a device
synchronize on both sides and the max over ranks.
"""

from __future__ import annotations

import time

import torch


def run_e2e(pipe, arena, cfg, args, rank: int, world: int, dev) -> dict:
    import torch.distributed as dist

    from quail_b200.api.session import run_filter_query
    from quail_b200.utils.synthetic import make_workload, rows_for_tokens

    wl = make_workload(rows_for_tokens(args.steps * args.chunk_tokens), seed=2000 + rank)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    result = run_filter_query(pipe, arena, wl, chunk_tokens=args.chunk_tokens)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    stats = result["stats"]
    t = torch.tensor([wall, float(wl.prompt_tokens()), float(wl.rows), float(stats.passes),
                      float(stats.h2d_bytes), float(stats.d2h_bytes)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        wall = float(mx[0])
    prompt, rows, passes, h2d, d2h = (float(v) for v in t[1:])
    return {"value": round(prompt / wall, 1), "unit": "prompt tokens/s", "rows_per_second": round(rows / wall, 1),
            "h2d_bytes_per_step": int(h2d / max(passes, 1)), "d2h_bytes_per_step": int(d2h / max(passes, 1)),
            "rows": int(rows), "passes": int(passes), "wall_s": round(wall, 3),
            "api": "quail_b200.api.session.run_filter_query (AI.IF region over a registered token table)"}
