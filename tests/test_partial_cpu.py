"""WHERE tests of an AI.MAP answer decided on the answer's text so far.

Unit checks of the decision rules (quail_b200.sql.partial), a soundness sweep
(a decided test has the decided value on every completion of the text so
far, evaluated by the executor's own Arrow evaluation), and the query end to
end on the fp32 tiny Qwen3: the same rows with and without the early stops,
fewer decode steps with them.
Reference: crates/quail-datafusion/src/derive/partial.rs tests (decisions
over completions) and quail/execution/answer_stops.py.
"""

import copy

import numpy as np
import pyarrow as pa
import pytest

import quail_b200 as quail
from quail_b200.sql import partial as Pt
from quail_b200.sql.executor import Executor, Relation, is_model_call, node_key, parse, walk


def _cond(where: str):
    e = parse(f"SELECT * FROM t WHERE {where}")["where"]
    call = next(n for n in walk(e) if is_model_call(n))
    return e, node_key(call)


def _decide(where, text, **kw):
    e, k = _cond(where)
    return Pt.decide(e, k, Pt.Completions(text, **kw), node_key)


M = "AI.MAP(body, 'Summarize', 16)"


@pytest.mark.parametrize("where,text,want", [
    (f"{M} LIKE 'Yes%'", "Ye", Pt.UNDECIDED),
    (f"{M} LIKE 'Yes%'", "Yes", Pt.TRUE),
    (f"{M} LIKE 'Yes%'", "No", Pt.NOT_TRUE),
    (f"{M} NOT LIKE 'Yes%'", "No", Pt.TRUE),
    (f"{M} ILIKE 'yes%'", "YES, it", Pt.TRUE),
    (f"{M} LIKE '%cat%'", "the cat", Pt.TRUE),
    (f"{M} LIKE '%cat%'", "the ca", Pt.UNDECIDED),
    (f"{M} LIKE 'a_c'", "abcd", Pt.NOT_TRUE),
    (f"{M} LIKE 'a_c'", "ab", Pt.UNDECIDED),
    (f"{M} = 'red'", "re", Pt.UNDECIDED),
    (f"{M} = 'red'", "bl", Pt.NOT_TRUE),
    (f"{M} = 'red'", "reddish", Pt.NOT_TRUE),
    (f"{M} <> 'red'", "bl", Pt.TRUE),
    (f"{M} IN ('red', 'green')", "g", Pt.UNDECIDED),
    (f"{M} IN ('red', 'green')", "b", Pt.NOT_TRUE),
    (f"{M} NOT IN ('red', 'green')", "b", Pt.TRUE),
    (f"LENGTH({M}) < 5", "abcd", Pt.UNDECIDED),
    (f"LENGTH({M}) < 5", "abcde", Pt.NOT_TRUE),
    (f"LENGTH({M}) >= 5", "abcde", Pt.TRUE),
    (f"LENGTH({M}) > 2 AND LENGTH({M}) < 4", "abcd", Pt.NOT_TRUE),
    (f"STARTS_WITH(LOWER({M}), 'pos')", "Posi", Pt.TRUE),
    (f"STARTS_WITH(LOWER({M}), 'pos')", "Neg", Pt.NOT_TRUE),
    (f"STARTS_WITH({M}, 'pos')", "po", Pt.UNDECIDED),
    (f"LEFT({M}, 3) = 'abc'", "abcz", Pt.TRUE),
    (f"LEFT({M}, 3) = 'abc'", "ab", Pt.UNDECIDED),
    (f"SUBSTR({M}, 1, 2) = 'ab'", "ax", Pt.NOT_TRUE),
    (f"UPPER({M}) = 'YES'", "yes", Pt.UNDECIDED),
    (f"UPPER({M}) = 'YES'", "yo", Pt.NOT_TRUE),
    (f"{M} < 'm'", "apple", Pt.TRUE),
    (f"{M} < 'm'", "zebra", Pt.NOT_TRUE),
    (f"{M} < 'ap'", "a", Pt.UNDECIDED),
    (f"{M} >= 'm'", "zeb", Pt.TRUE),
    (f"{M} IS NULL", "x", Pt.NOT_TRUE),
    (f"{M} IS NOT NULL", "", Pt.TRUE),
    (f"NOT ({M} LIKE 'a%')", "b", Pt.TRUE),
    (f"{M} LIKE 'a%' OR LENGTH({M}) > 3", "bcde", Pt.TRUE),
    (f"{M} LIKE 'a%' OR LENGTH({M}) > 3", "bc", Pt.UNDECIDED),
    (f"COALESCE({M}, 'x') = 'y'", "y", Pt.UNDECIDED),      # no rule: never decided
])
def test_decisions(where, text, want):
    assert _decide(where, text) == want


def test_complete_answers_are_decided_exactly():
    assert _decide(f"{M} = 'red'", "red", complete=True) == Pt.TRUE
    assert _decide(f"{M} = 'red'", "re", complete=True) == Pt.NOT_TRUE
    assert _decide(f"LENGTH({M}) < 5", "abcd", complete=True) == Pt.TRUE
    assert _decide(f"{M} LIKE 'a_c'", "abc", complete=True) == Pt.TRUE


def test_a_bounded_answer_is_decided_sooner():
    # at most two more characters: 'ab' can no longer reach five
    assert _decide(f"LENGTH({M}) >= 5", "ab", max_chars=2) == Pt.NOT_TRUE
    assert _decide(f"LENGTH({M}) >= 5", "ab") == Pt.UNDECIDED


def test_reads_answer_alone():
    e, k = _cond(f"LOWER({M}) LIKE 'y%'")
    assert Pt.reads_answer_alone(e, k, node_key)
    e, k = _cond(f"{M} = title")
    assert not Pt.reads_answer_alone(e, k, node_key)


def _eval_with(where: str, answers: list):
    """The condition on each answer, by the executor's own evaluation (the call -> a column)."""
    e, k = _cond(where)
    e = copy.deepcopy(e)

    def sub(n):
        if isinstance(n, dict):
            for kk, v in list(n.items()):
                if isinstance(v, dict) and v.get("type") == "call" and node_key(v) == k:
                    n[kk] = {"type": "column", "name": "ans"}
                else:
                    sub(v)
        elif isinstance(n, list):
            for i, v in enumerate(n):
                if isinstance(v, dict) and v.get("type") == "call" and node_key(v) == k:
                    n[i] = {"type": "column", "name": "ans"}
                else:
                    sub(v)
    sub(e)
    ex = Executor({}, None)
    rel = Relation.from_table(pa.table({"ans": pa.array(answers, pa.string())}), None)
    return ex.eval(e, rel).to_pylist()


SWEEP = [f"{M} LIKE 'ab%'", f"{M} LIKE '%b_'", f"{M} ILIKE 'A%c'", f"{M} = 'abc'", f"{M} <> 'ab'",
         f"{M} IN ('a', 'abc', 'ba')", f"LENGTH({M}) < 3", f"LENGTH({M}) BETWEEN 2 AND 3",
         f"STARTS_WITH(UPPER({M}), 'AB')", f"LEFT({M}, 2) = 'ab'", f"{M} < 'b'", f"{M} >= 'ab'",
         f"NOT ({M} LIKE 'b%') AND LENGTH({M}) > 1", f"{M} LIKE 'a%' OR {M} LIKE 'c%'"]


@pytest.mark.parametrize("where", SWEEP)
def test_decisions_hold_for_every_completion(where):
    rng = np.random.default_rng(len(where))
    alphabet = list("abcAB")
    prefixes = [""] + ["".join(rng.choice(alphabet, int(rng.integers(1, 5)))) for _ in range(40)]
    for w in prefixes:
        d = _decide(where, w)
        if d == Pt.UNDECIDED:
            continue
        tails = [""] + ["".join(rng.choice(alphabet, int(rng.integers(1, 6)))) for _ in range(30)]
        got = _eval_with(where, [w + t for t in tails])
        if d == Pt.TRUE:
            assert all(v is True for v in got), (where, w, got)
        else:
            assert not any(v is True for v in got), (where, w, got)


def _table(n=16, seed=0):
    rng = np.random.default_rng(seed)
    words = ["ending", "music", "cast", "plot", "money", "great", "bad", "long", "short", "story"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 10)))) for _ in range(n)]
    return pa.table({"id": list(range(n)), "body": bodies})


def test_map_answers_stop_once_the_test_is_decided():
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=256)
    with quail.Session(config=cfg) as s:
        s.register("t", quail.DocumentProvider.from_table(_table(), id_col="id"))
        # the random model's tokens are mostly outside the byte tokenizer's range (they decode
        # to nothing): read every token as one letter so the answers have text to test
        tok = s.engine().tokenizer
        tok.decode = lambda ids: "".join(chr(97 + int(i) % 7) for i in ids)
        full = s.sql(f"SELECT id, {M} AS m FROM t ORDER BY id").collect().to_pylist()
        k = min(3, min(len(r["m"]) for r in full))
        first = full[0]["m"][:1]
        for where in (f"LENGTH({M}) < {k}", f"LEFT({M}, 1) = '{first}'" if first not in ("'", "\\") else None):
            if where is None:
                continue
            want = sorted(r["id"] for r in full if _eval_with(where, [r["m"]])[0])
            on = s.sql(f"SELECT id FROM t WHERE {where}").run()
            s.sql("SET quail.pushdown = false").run()
            off = s.sql(f"SELECT id FROM t WHERE {where}").run()
            s.sql("SET quail.pushdown = true").run()
            assert sorted(on.table.column("id").to_pylist()) == want
            assert sorted(off.table.column("id").to_pylist()) == want
            assert on.report.get("stopped_early", 0) > 0
            assert "stopped_early" not in off.report
            assert on.report["fresh_tokens"] < off.report["fresh_tokens"]


def test_extraction_field_and_prefix_rules():
    e, k = _cond("AI.EXTRACT(body, {'year': 'Which year?'})['year'] LIKE '2027%'")
    assert Pt.extraction_field(e, k, node_key) == "year"
    # an extraction may still answer NULL: a test is only ever decided NOT TRUE
    assert Pt.decide(e, k, Pt.Completions("2027", may_be_null=True), node_key, "year") == Pt.UNDECIDED
    assert Pt.decide(e, k, Pt.Completions("2026", may_be_null=True), node_key, "year") == Pt.NOT_TRUE
    e2, k2 = _cond("AI.EXTRACT(body, {'a': 'A?', 'b': 'B?'})['a'] = AI.EXTRACT(body, {'a': 'A?', 'b': 'B?'})['b']")
    assert Pt.extraction_field(e2, k2, node_key) is None          # two fields: no single answer to stop
    assert Pt.extraction_prefix("  Phr") is None                  # may still be the "Phrase:" label
    assert Pt.extraction_prefix("Phrase: 2027 ") == "2027"
    assert Pt.extraction_prefix(" the end ") == "the end"


def test_extraction_stop_wiring():
    """The executor attaches the WHERE test to the one question whose field it reads, and that
    question's decode gets a test of its text so far."""
    from quail_b200.sql.executor import BoundCall, _stop_test
    x = "AI.EXTRACT(body, {'who': 'Who?', 'year': 'Which year?'})"
    e, k = _cond(f"{x}['year'] LIKE '2027%'")
    ex = Executor({}, None)
    ex.call_counts = {k: 1}
    stops = ex._answer_stops(e)
    assert stops[k]["field"] == "year" and stops[k]["test"] is e
    b = BoundCall(key=f"{k}#1", kind="extract", preamble="", tail="", doc_expr={}, stop={**stops[k], "call": k})
    test = _stop_test(b)
    assert test("Phrase: 2026") == Pt.NOT_TRUE
    assert test(" 20") == Pt.UNDECIDED and test("Phra") == Pt.UNDECIDED
    e2, k2 = _cond(f"{x}['year'] = {x}['who']")
    ex.call_counts = {k2: 2}
    assert ex._answer_stops(e2) == {}
