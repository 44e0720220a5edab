"""Measured metrics of a query: per model region ("node"), merged across workers.

The metric names and the merge rule are the reference's report
(crates/quail/src/report.rs:24-39, 240-262, 355-380): every count adds across
workers; a worker's peak memory is its own, so the largest is kept; workers
run side by side, so a region's wall time is the slowest worker's.
"""

from __future__ import annotations

# the per-node metrics, in the order a report lists them
METRICS = ("wall_s", "input_rows", "output_rows", "evaluated_documents", "evaluated_document_pairs",
           "fresh_tokens", "cached_tokens", "kv_hits", "kv_misses", "kv_removals", "kv_recomputations",
           "peak_gpu_bytes", "gpu_s", "chunks")
_LARGEST = ("peak_gpu_bytes", "wall_s")
# region stats the session reads besides the metrics
_COUNTS = ("passes", "fresh_tokens", "documents", "asked", "cached_tokens", "kv_hits", "kv_misses", "kv_removals",
           "kv_recomputations", "gpu_s", "chunks", "output_rows", "reused_documents", "replays",
           "evaluated_document_pairs")


def merge_worker_stats(parts: list, counted: list, rows: int) -> dict:
    """One region's stats from its workers' stats. `counted[i]` says whether worker i's counts
    add (the other ranks of a tensor-parallel copy repeat rank 0's work); the largest
    peak and wall time are taken over every worker."""
    out = {"rows": rows, "per_worker": list(parts)}
    for k in _COUNTS:
        out[k] = 0
    for st, c in zip(parts, counted):
        if not c:
            continue
        for k in _COUNTS:
            out[k] += st.get(k, 0)
    for k in _LARGEST:
        out[k] = max((st.get(k, 0) for st in parts), default=0)
    out["input_rows"] = rows
    return out


def node_metrics(stats: dict) -> dict:
    """A region's stats under the report's metric names."""
    m = {k: stats.get(k, 0) for k in METRICS}
    m["evaluated_documents"] = stats.get("documents", 0)
    m["input_rows"] = stats.get("input_rows", stats.get("rows", 0))
    return m


def totals(nodes: dict) -> dict:
    """The whole query's metrics: sums over its nodes, the largest peak."""
    out = {k: 0 for k in METRICS}
    for m in nodes.values():
        for k in METRICS:
            if k == "peak_gpu_bytes":
                out[k] = max(out[k], m.get(k, 0))
            else:
                out[k] += m.get(k, 0)
    return out
