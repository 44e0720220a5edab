"""Demand rules, transcript style: the rows stay the same, the questions asked drop.

Each query runs twice over the same table, through the real parser and
executor with the oracle engine (tests/oracle.py): once with the demand
rules (CASE guards, AND / OR guards, fetch for LIMIT) and once with
`SET quail.pushdown = false`, which asks every call on every row that
reaches its operator. Both runs must return the same rows; the transcript
records "asked k of n" for both and must equal the committed one
(QUAIL_UPDATE_TRANSCRIPTS=1 rewrites it). Reference discipline:
tests/helpers/transcript.py, tests/planner/test_guards.py.
"""

import os

import numpy as np
import pyarrow as pa
import pytest

import quail_b200 as quail
from oracle import OracleEngine

HERE = os.path.dirname(os.path.abspath(__file__))
TRANSCRIPTS = os.path.join(HERE, "fixtures", "transcripts")
IF_ENDING = "AI.IF(PROMPT('Does the review discuss the ending? {0}', body))"
SCORE_POS = "AI.SCORE(PROMPT('Is the review positive? {0}', body))"
KINDS = "AI.CLASSIFY(body, ['praise', 'complaint', 'neutral remark'])"
CFG = quail.EngineConfig(model="qwen3-tiny", device="cpu")


def _table(n=200, seed=0):
    rng = np.random.default_rng(seed)
    words = ["ending", "music", "cast", "plot", "money", "great", "bad", "long", "short", "story"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 12)))) for _ in range(n)]
    return pa.table({"id": list(range(n)), "body": bodies, "stars": [int(x) for x in rng.integers(1, 6, n)]})


def _run(sql: str, pushdown: bool):
    oracle = OracleEngine()
    s = quail.Session(config=CFG)
    s.register("reviews", quail.DocumentProvider.from_table(_table(), id_col="id"))
    s.attach_engine(oracle)
    if not pushdown:
        s.sql("SET quail.pushdown = false").run()
    rows = s.sql(sql).collect()
    return rows, len(oracle.asked), oracle


CASES = {
    "case_guard": f"SELECT id, CASE WHEN {IF_ENDING} THEN {SCORE_POS} END AS s FROM reviews ORDER BY id",
    "case_else_guard": (f"SELECT id, CASE WHEN {IF_ENDING} THEN {KINDS} ELSE 'none' END AS k FROM reviews "
                        "ORDER BY id"),
    "case_column_guard": f"SELECT id, CASE WHEN stars >= 4 THEN {SCORE_POS} ELSE 0.0 END AS s FROM reviews",
    "or_guard": f"SELECT id FROM reviews WHERE stars = 5 OR {IF_ENDING}",
    "and_inside_or": f"SELECT id FROM reviews WHERE (stars > 2 AND {IF_ENDING}) OR stars = 1",
    "projection_and": f"SELECT id, {IF_ENDING} AND {SCORE_POS} > 0.5 AS both FROM reviews",
    "iff_guard": f"SELECT id, IFF(stars > 3, {SCORE_POS}, NULL) AS s FROM reviews",
    "limit_fetch": f"SELECT id FROM reviews WHERE {IF_ENDING} LIMIT 10",
    "limit_offset_fetch": f"SELECT id, body FROM reviews WHERE {IF_ENDING} LIMIT 5 OFFSET 7",
    "order_limit_fetch": f"SELECT id FROM reviews WHERE {IF_ENDING} ORDER BY stars DESC, id LIMIT 8",
    "guarded_classify_after_filter": (f"SELECT id, CASE WHEN {SCORE_POS} > 0.5 THEN {KINDS} END AS k "
                                      f"FROM reviews WHERE {IF_ENDING}"),
}


def _transcript(name, sql, on_rows, on_asked, off_asked, n_rows):
    lines = [f"-- {name}", sql.strip(), f"rows: {on_rows.num_rows}",
             f"asked {on_asked} of {off_asked} questions with the demand rules on ({n_rows} table rows)"]
    for r in on_rows.slice(0, 5).to_pylist():
        lines.append("  " + ", ".join(f"{k}={v!r}" for k, v in r.items()))
    return "\n".join(lines) + "\n"


@pytest.mark.parametrize("name", sorted(CASES))
def test_demand_rules_keep_rows_and_ask_less(name):
    sql = CASES[name]
    on_rows, on_asked, _ = _run(sql, True)
    off_rows, off_asked, _ = _run(sql, False)
    assert on_rows.equals(off_rows), (name, on_rows.to_pylist()[:5], off_rows.to_pylist()[:5])
    assert on_asked < off_asked, (name, on_asked, off_asked)
    text = _transcript(name, sql, on_rows, on_asked, off_asked, 200)
    path = os.path.join(TRANSCRIPTS, f"{name}.txt")
    if os.environ.get("QUAIL_UPDATE_TRANSCRIPTS") == "1" or not os.path.exists(path):
        with open(path, "w") as f:
            f.write(text)
    with open(path) as f:
        assert f.read() == text


def test_case_guard_asks_the_score_only_where_the_filter_holds():
    rows, asked, oracle = _run(CASES["case_guard"], True)
    ifs = [a for a in oracle.asked if a[0] == "filter"]
    scores = [a for a in oracle.asked if a[0] == "score"]
    assert len(ifs) == 200
    kept = sum(1 for v in rows.column("s").to_pylist() if v is not None)
    assert len(scores) == kept and 0 < kept < 200


def test_limit_stops_asking_once_enough_rows_passed():
    rows, asked, _ = _run(CASES["limit_fetch"], True)
    assert rows.num_rows == 10
    assert asked < 200 * 0.6


def test_stream_yields_rows_before_the_table_is_done():
    oracle = OracleEngine()
    s = quail.Session(config=CFG)
    s.register("reviews", quail.DocumentProvider.from_table(_table(3000, seed=3), id_col="id"))
    s.attach_engine(oracle)
    reader = s.sql(f"SELECT id FROM reviews WHERE {IF_ENDING}").execute_stream(batch_rows=64)
    first = reader.read_next_batch()
    assert first.num_rows <= 64
    assert len(oracle.asked) < 3000          # only the first slice was asked so far
    rest = reader.read_all()
    got = first.column(0).to_pylist() + rest.column(0).to_pylist()
    whole, _, _ = _run_on(3000, 3, f"SELECT id FROM reviews WHERE {IF_ENDING}")
    assert got == whole.column("id").to_pylist()


def test_stream_limit_is_a_fetch_demand():
    oracle = OracleEngine()
    s = quail.Session(config=CFG)
    s.register("reviews", quail.DocumentProvider.from_table(_table(3000, seed=3), id_col="id"))
    s.attach_engine(oracle)
    got = s.sql(f"SELECT id FROM reviews WHERE {IF_ENDING}").execute_stream(batch_rows=64, limit=20).read_all()
    assert got.num_rows == 20
    assert len(oracle.asked) < 200


def _run_on(n, seed, sql):
    oracle = OracleEngine()
    s = quail.Session(config=CFG)
    s.register("reviews", quail.DocumentProvider.from_table(_table(n, seed=seed), id_col="id"))
    s.attach_engine(oracle)
    return s.sql(sql).collect(), len(oracle.asked), oracle


def test_distinct_over_the_key_keeps_the_limit_fetch():
    """DISTINCT with the table's id column removes no row: the LIMIT still stops the model early."""
    sql = f"SELECT DISTINCT id, stars FROM reviews WHERE {IF_ENDING} LIMIT 6"
    on, asked_on, _ = _run(sql, pushdown=True)
    off, asked_off, _ = _run(sql, pushdown=False)
    assert on.num_rows == 6 and on.to_pylist() == off.to_pylist()
    assert asked_on < asked_off
    # without the key the DISTINCT may merge rows: every row is asked
    _, asked_nokey, _ = _run(f"SELECT DISTINCT stars FROM reviews WHERE {IF_ENDING} LIMIT 3", pushdown=True)
    assert asked_nokey == asked_off
