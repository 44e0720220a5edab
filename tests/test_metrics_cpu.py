"""Query metrics: per model region ("node"), merged across workers, and the whole query's.

The names and the merge rule are the reference's report (crates/quail/src/report.rs:24-39,
240-262, 355-380): counts add across workers, the peak is the largest.
"""

import pyarrow as pa

import quail_b200 as quail
from quail_b200.runtime.report import METRICS, merge_worker_stats, node_metrics, totals


def _session():
    s = quail.Session(config=quail.EngineConfig(model="qwen3-tiny", device="cpu"))
    t = pa.table({"id": list(range(6)), "body": ["a long review of the plot", "great music", "bad ending",
                                                 "short", "money talk", "a long review of the plot"]})
    s.register("r", quail.DocumentProvider.from_table(t, id_col="id"))
    return s


def test_every_region_reports_the_node_metrics():
    with _session() as s:
        res = s.sql("SELECT id, AI.SCORE(PROMPT('Is {0} positive?', body)) AS p FROM r "
                    "WHERE AI.IF(PROMPT('Is {0} about music or plot?', body), {'selectivity': 0.9})").run()
        rep = res.report
    nodes = rep["node_metrics"]
    regions = [k for k in nodes if k != "output"]
    assert regions and all(set(METRICS) <= set(nodes[k]) for k in regions)
    first = nodes[regions[0]]
    # six rows, five distinct documents: each distinct document is computed once (a miss)
    assert first["input_rows"] == 6 and first["evaluated_documents"] == 5 and first["kv_misses"] == 5
    # every document and follow-up question read the shared instruction prefix from the arena
    assert first["cached_tokens"] > 0 and rep["cached_tokens"] >= first["cached_tokens"]
    assert first["chunks"] >= 1 and first["peak_gpu_bytes"] == 0 and first["wall_s"] > 0
    assert nodes["output"]["output_rows"] == res.table.num_rows
    assert rep["peak_gib"] == 0.0 and rep["usd_per_query"] is None    # the host has no hourly price here
    assert rep["fresh_tokens"] == sum(nodes[k]["fresh_tokens"] for k in regions)


def test_explain_analyze_lists_the_measured_nodes():
    with _session() as s:
        text = s.sql("SELECT id FROM r WHERE AI.IF(PROMPT('Is {0} short?', body))").explain(analyze=True)
    assert "measured:" in text and "cached_tokens=" in text
    assert "quail.region[filter]" in text and "kv_misses=" in text


def test_worker_stats_add_counts_and_keep_the_largest_peak():
    a = {"passes": 3, "fresh_tokens": 100, "documents": 4, "asked": 4, "cached_tokens": 40, "kv_hits": 1,
         "peak_gpu_bytes": 7 << 30, "wall_s": 2.0, "gpu_s": 1.5}
    b = {"passes": 2, "fresh_tokens": 60, "documents": 3, "asked": 3, "cached_tokens": 30, "kv_hits": 0,
         "peak_gpu_bytes": 9 << 30, "wall_s": 3.0, "gpu_s": 1.0}
    m = merge_worker_stats([a, b], [True, True], rows=9)
    assert (m["passes"], m["fresh_tokens"], m["documents"], m["cached_tokens"], m["kv_hits"]) == (5, 160, 7, 70, 1)
    assert m["peak_gpu_bytes"] == 9 << 30 and m["wall_s"] == 3.0 and m["gpu_s"] == 2.5
    assert m["input_rows"] == 9 and len(m["per_worker"]) == 2
    # the second rank of a tensor-parallel copy repeats rank 0's counts: only its peak is read
    tp = merge_worker_stats([a, b], [True, False], rows=4)
    assert tp["fresh_tokens"] == 100 and tp["peak_gpu_bytes"] == 9 << 30
    n1, n2 = node_metrics(m), node_metrics(tp)
    assert n1["evaluated_documents"] == 7
    tot = totals({"x": n1, "y": n2})
    assert tot["fresh_tokens"] == 260 and tot["peak_gpu_bytes"] == 9 << 30


def test_kv_pool_cap_and_answer_admission_flags(monkeypatch, tmp_path):
    import json
    import os

    import pytest

    from quail_b200.api.config import EngineConfig
    from quail_b200.api.engine import CallSpec, ModelEngine
    from quail_b200.engine.stage_executor import answer_admission_mode
    from quail_b200.models.config import QWEN3_TINY
    from quail_b200.planner.budgets import Budgets
    full = Budgets.for_model(QWEN3_TINY, "cpu").arena_pages(16)
    monkeypatch.setenv("QUAIL_KV_POOL_TOKENS", "4096")
    assert Budgets.for_model(QWEN3_TINY, "cpu").arena_pages(16) == min(full, 256)
    monkeypatch.delenv("QUAIL_KV_POOL_TOKENS")
    monkeypatch.setenv("QUAIL_ANSWER_ADMISSION", "sometimes")
    with pytest.raises(ValueError, match="QUAIL_ANSWER_ADMISSION"):
        answer_admission_mode()
    docs = ["one two three four", "five six seven", "eight nine"]
    calls = [CallSpec(kind="map", tail="\nSummarize:", name="m", max_tokens=6)]
    got = {}
    for mode in ("headroom", "headroom=0"):
        monkeypatch.setenv("QUAIL_ANSWER_ADMISSION", mode)
        monkeypatch.setenv("QUAIL_HEADROOM_TRACE", str(tmp_path / mode))
        eng = ModelEngine(EngineConfig(model="qwen3-tiny", device="cpu"), pages=64)
        assert eng.executor.answer_headroom == (mode == "headroom")
        got[mode] = eng.run_region("Instruction:\n", docs, calls).values
        files = os.listdir(tmp_path / mode)
        assert len(files) == 1
        trace = json.load(open(tmp_path / mode / files[0]))
        assert trace["answer_admission"] == mode and trace["num_pages"] == 64
        assert trace["samples"] and all(s[3] + s[4] == 64 for s in trace["samples"])
    # the admission rule changes when work starts, never the answers
    assert got["headroom"] == got["headroom=0"]


def test_documents_are_tokenized_once_per_session():
    with _session() as s:
        s.sql("SELECT id FROM r WHERE AI.IF(PROMPT('Is {0} short?', body))").collect()
        store = s.engine().token_store
        misses = store.misses
        assert misses == 5 and store.hits == 0          # five distinct bodies
        s.sql("SELECT id, AI.SCORE(PROMPT('Is {0} long?', body)) AS p FROM r").collect()
        assert store.misses == misses and store.hits >= 5
        assert store.mean_tokens(["great music", "bad ending"]) > 0
    from quail_b200.engine.token_store import TokenStore
    small = TokenStore(capacity_tokens=3)
    small.put("a", [1, 2])
    small.put("b", [3, 4])
    assert small.get("a") is None and len(small) == 1   # the oldest went out
