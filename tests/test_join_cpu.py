"""AI joins as pair questions that share the anchor side's document.

A 20 x 20 AI join asks 400 pair questions. With the demand rules on, each
anchor document is prefilled once and read by its 20 pairs; with them off,
every pair carries its own copy of the anchor document. The prompts are the
same token for token, so the rows must be equal; the fresh tokens must drop.
Reference: quail/backends/quail/executor/operators/join.py:47-739 (pair
lists, shared anchor KV), crates/quail-planner/src/search.rs:891 (anchors).
"""

import numpy as np
import pyarrow as pa
import pytest

import quail_b200 as quail
from oracle import OracleEngine
from quail_b200.planner.search import choose_anchor, join_costs, order_filters

JOIN = ("SELECT a.id AS a_id, b.id AS b_id FROM a JOIN b "
        "ON AI.IF(PROMPT('Is {0} about the same thing as {1}?', a.txt, b.txt)) ORDER BY a_id, b_id")


def _tables(na=20, nb=20, seed=0, long_side="a"):
    rng = np.random.default_rng(seed)
    words = ["refund", "late", "broken", "great", "thanks", "order", "ending", "cast", "plot", "music"]

    def body(lo, hi):
        return " ".join(rng.choice(words, size=int(rng.integers(lo, hi))))
    la, lb = ((40, 80), (3, 8)) if long_side == "a" else ((3, 8), (40, 80))
    a = pa.table({"id": list(range(na)), "txt": [body(*la) for _ in range(na)]})
    b = pa.table({"id": list(range(nb)), "txt": [body(*lb) for _ in range(nb)]})
    return a, b


def _session(cfg, a, b, engine=None, pushdown=True):
    s = quail.Session(config=cfg)
    s.register("a", a)
    s.register("b", b)
    if engine is not None:
        s.attach_engine(engine)
    if not pushdown:
        s.settings["quail.pushdown"] = "false"
    return s


def test_pair_join_shares_anchor_documents_on_the_oracle():
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu")
    a, b = _tables()
    on, off = OracleEngine(), OracleEngine()
    rows_on = _session(cfg, a, b, on).sql(JOIN).run()
    rows_off = _session(cfg, a, b, off, pushdown=False).sql(JOIN).run()
    assert rows_on.table.equals(rows_off.table)
    assert 0 < rows_on.table.num_rows < 400
    assert len(on.asked) == len(off.asked) == 400          # every pair asked once either way
    assert rows_on.report["evaluated_documents"] == 20     # anchors prefilled once each
    assert rows_off.report["evaluated_documents"] == 400
    assert rows_on.report["joins"] == [{"anchor": "left"}]  # the long documents are the anchors


def test_the_anchor_is_the_side_that_saves_tokens():
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu")
    a, b = _tables(long_side="b")
    res = _session(cfg, a, b, OracleEngine()).sql(JOIN).run()
    assert res.report["joins"] == [{"anchor": "right"}]
    forced = JOIN.replace("a.txt, b.txt))", "a.txt, b.txt), {'anchor': 'left'})")
    res2 = _session(cfg, a, b, OracleEngine()).sql(forced).run()
    assert res2.report["joins"] == [{"anchor": "left"}]


def test_join_cost_and_filter_order_rules():
    left = ["x" * 400] * 3 + ["y" * 400] * 3          # 2 distinct long documents, 6 pairs
    right = ["z" * 8] * 6
    cl, cr = join_costs(left, right)
    assert cl < cr and choose_anchor(left, right) == "L"
    assert choose_anchor(left, right, "right") == "R"
    # equal cost: the more selective first; equal selectivity: the cheaper first
    assert order_filters([10, 10], [0.9, 0.1]) == [1, 0]
    assert order_filters([40, 10], [0.5, 0.5]) == [1, 0]
    # a costly but very selective filter can still go first
    assert order_filters([30, 10], [0.05, 0.9]) == [0, 1]


@pytest.mark.slow
def test_pair_join_on_the_tiny_model_prefills_each_anchor_once():
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=512)
    a, b = _tables(8, 6, seed=2)
    with _session(cfg, a, b) as s:
        on = s.sql(JOIN).run()
        s.settings["quail.pushdown"] = "false"
        off = s.sql(JOIN).run()
    assert on.table.equals(off.table)
    assert on.report["asked"] == off.report["asked"] == 48
    assert on.report["fresh_tokens"] < 0.7 * off.report["fresh_tokens"]
