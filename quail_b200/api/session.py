"""Session entry points (filled in by the SQL front end)."""

from __future__ import annotations


def run_filter_query(pipe, arena, workload, *, chunk_tokens: int = 16384, name: str = "if"):
    """Run `SELECT ... WHERE AI.IF(PROMPT(<instruction> {0}, body))` over a token table.

    `workload` holds the tokenized template prefix, the question suffix and
    one body per row. Returns the kept row indices and executor stats.
    """
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor

    rows = pipe.w.answer_rows.shape[0]
    half = rows // 2
    ex = StageExecutor(pipe, arena, chunk_tokens)
    call = Call(kind="filter", suffix=workload.suffix, true_cols=list(range(half)),
                false_cols=list(range(half, rows)), name=name)
    results = RegionRun(ex, workload.prefix, workload.bodies, [call]).run()
    kept = [i for i, r in enumerate(results) if r.values.get(name)]
    return {"kept": kept, "stats": ex.stats, "results": results}
