"""A call the WHERE clause already answered on every row is read, not asked again.

The same AI call written in the WHERE clause and in the SELECT list (or in two
conjuncts) is asked once per row: the answers of a conjunct computed on every
row (no demand guard) travel with the rows the filter keeps. A call the WHERE
clause asked under a guard (an OR) is asked again where the SELECT list needs
it. Rows match the run with the demand rules off.
Reference: crates/quail-datafusion/src/rules/repeated.rs (MergeRepeatedAiCalls).
"""

import numpy as np
import pyarrow as pa

import quail_b200 as quail
from oracle import OracleEngine

KIND = "AI.CLASSIFY(body, ['praise', 'complaint', 'neutral remark'])"
MAP = "AI.MAP(body, 'Name the topic.', 8)"


def _table(n=60, seed=3):
    rng = np.random.default_rng(seed)
    words = ["ending", "music", "cast", "plot", "money", "great", "bad", "long", "short", "story"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 12)))) for _ in range(n)]
    return pa.table({"id": list(range(n)), "body": bodies, "stars": [int(x) for x in rng.integers(1, 6, n)]})


def _run(sql, pushdown=True):
    oracle = OracleEngine()
    s = quail.Session(config=quail.EngineConfig(model="qwen3-tiny", device="cpu"))
    s.register("reviews", quail.DocumentProvider.from_table(_table(), id_col="id"))
    s.attach_engine(oracle)
    if not pushdown:
        s.sql("SET quail.pushdown = false").run()
    return s.sql(sql).collect().to_pylist(), oracle.asked


def test_where_and_select_ask_once():
    sql = f"SELECT id, {KIND} AS k FROM reviews WHERE {KIND} <> 'praise' ORDER BY id"
    rows, asked = _run(sql)
    assert len(asked) == 60
    assert rows and all(r["k"] != "praise" for r in rows)
    rows_off, _ = _run(sql, pushdown=False)
    assert rows == rows_off


def test_two_conjuncts_ask_once():
    sql = f"SELECT id FROM reviews WHERE {MAP} <> 'answer-1' AND LENGTH({MAP}) > 3 ORDER BY id"
    rows, asked = _run(sql)
    assert len(asked) == 60
    assert rows == _run(sql, pushdown=False)[0]


def test_guarded_where_answer_is_asked_again_where_needed():
    sql = f"SELECT id, {KIND} AS k FROM reviews WHERE stars = 5 OR {KIND} = 'complaint' ORDER BY id"
    rows, asked = _run(sql)
    on = len(asked)
    rows_off, asked_off = _run(sql, pushdown=False)
    assert rows == rows_off
    assert all(r["k"] is not None for r in rows)
    assert on <= len(asked_off)
