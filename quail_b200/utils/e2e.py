"""End-to-end timing of the flagship query through the public API.

The timed region is one `Session.sql(...).run()` of

    SELECT id FROM docs WHERE AI.IF(PROMPT('<16-word instruction> {0}', body))

over a registered table of synthetic token-id bodies (by default the
configuration's 200,000 rows, sharded over the ranks): SQL parsing and
planning, prompt tokenization, chunk packing on the host, each chunk's
host->device copy from pinned memory, the forward passes, and the
device->host copy of every chunk's answers, wall-clock with a device
synchronize on both sides; the max over ranks.
"""

from __future__ import annotations

import time

import numpy as np
import pyarrow as pa
import torch

INSTRUCTION = ("Does this document describe a product defect that a customer reported after using the item "
               "for several weeks")


def run_e2e(pipe, arena, cfg, args, rank: int, world: int, dev) -> dict:
    import torch.distributed as dist

    import quail_b200 as quail
    from quail_b200.api.engine import ModelEngine
    from quail_b200.utils.synthetic import make_workload, rows_for_tokens

    total = getattr(args, "e2e_rows", None)
    if total:
        # the configuration's table, sharded over the ranks (each rank its 1/N of the rows)
        rows = total // world + (1 if rank < total % world else 0)
    else:
        rows = rows_for_tokens(args.steps * args.chunk_tokens)
    wl = make_workload(rows, seed=2000 + rank)
    lens = np.fromiter((len(b) for b in wl.bodies), dtype=np.int64, count=len(wl.bodies))
    offsets = np.zeros(len(lens) + 1, dtype=np.int32)
    np.cumsum(lens, out=offsets[1:])
    flat = np.concatenate(wl.bodies) if wl.bodies else np.zeros(0, np.int32)
    table = pa.table({"id": np.arange(wl.rows, dtype=np.int64),
                      "body": pa.ListArray.from_arrays(pa.array(offsets), pa.array(flat, pa.int32()))})
    config = quail.EngineConfig(model=args.model, device="b200", chunk_tokens=args.chunk_tokens, tokenizer="words")
    session = quail.Session(config=config)
    engine = ModelEngine.from_replica(config, pipe, arena)
    session.attach_engine(engine)
    session.register("docs", table)
    query = session.sql(f"SELECT id FROM docs WHERE AI.IF(PROMPT('{INSTRUCTION} {{0}}', body))")
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    result = query.run()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    st = engine.executor.stats
    tok = engine.tokenizer
    from quail_b200.api.prompts import bind_prompt
    bp = bind_prompt(f"{INSTRUCTION} {{0}}")
    per_row = len(tok.encode(bp.preamble)) + len(tok.encode(bp.tail))
    prompt_tokens = sum(len(b) for b in wl.bodies) + per_row * wl.rows
    t = torch.tensor([wall, float(prompt_tokens), float(wl.rows), float(st.passes), float(st.h2d_bytes),
                      float(st.d2h_bytes), float(result.table.num_rows)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        wall = float(mx[0])
    prompt, rows, passes, h2d, d2h, kept = (float(v) for v in t[1:])
    return {"value": round(prompt / wall, 1), "unit": "prompt tokens/s", "rows_per_second": round(rows / wall, 1),
            "h2d_bytes_per_step": int(h2d / max(passes, 1)), "d2h_bytes_per_step": int(d2h / max(passes, 1)),
            "rows": int(rows), "kept_rows": int(kept), "passes": int(passes), "wall_s": round(wall, 3),
            "table_rows": int(total) if total else int(rows),
            "api": "quail_b200.Session.sql(\"SELECT id FROM docs WHERE AI.IF(PROMPT(...))\").run()"}
