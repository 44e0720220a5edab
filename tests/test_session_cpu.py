"""The query API end to end on CPU: SQL -> plan -> regions on the fp32 tiny Qwen3.

This is the benchmark's CPU plumbing configuration: a 2-layer, hidden-256
Qwen3-architecture model (4 q / 2 kv heads, head_dim 64, SwiGLU 768, vocab
151936, random init) answering AI calls over small tables. The checks are
the SQL semantics: a filter keeps exactly the rows the model answers TRUE
for when asked alone, relational predicates run before the model, later
calls only see the rows earlier filters kept, and results are identical
whatever the chunk size.
"""

import numpy as np
import pyarrow as pa
import pytest

import quail_b200 as quail
from quail_b200.api.engine import CallSpec, ModelEngine
from quail_b200.api.prompts import bind_prompt


def _table(n=24, seed=0):
    rng = np.random.default_rng(seed)
    words = ["ending", "music", "cast", "plot", "money", "great", "bad", "long", "short", "story"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 12)))) for _ in range(n)]
    return pa.table({"id": list(range(n)), "body": bodies, "grp": [i % 3 for i in range(n)]})


@pytest.fixture(scope="module")
def session():
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=256)
    with quail.Session(config=cfg) as s:
        s.register("reviews", quail.DocumentProvider.from_table(_table(), id_col="id"))
        yield s


def _asked_alone(engine: ModelEngine, template: str, docs):
    bp = bind_prompt(template)
    out = engine.run_region(bp.preamble, docs, [CallSpec(kind="filter", tail=bp.tail, name="f")])
    return [v["f"] for v in out.values]


def test_filter_keeps_the_rows_the_model_answers_true(session):
    q = "SELECT r.id FROM reviews r WHERE AI.IF(PROMPT('Does the review discuss the ending? {0}', r.body))"
    got = session.sql(q).collect().column("id").to_pylist()
    t = _table()
    alone = _asked_alone(session.engine(), "Does the review discuss the ending? {0}", t.column("body").to_pylist())
    assert got == [i for i, keep in zip(t.column("id").to_pylist(), alone) if keep]


def test_relational_predicate_runs_before_the_model(session):
    r = session.sql("SELECT id FROM reviews WHERE grp = 1 AND AI.IF(PROMPT('Is it long? {0}', body))").run()
    assert r.report["evaluated_documents"] <= 8
    assert all(i % 3 == 1 for i in r.table.column("id").to_pylist())


def test_score_classify_and_guards(session):
    q = """
        SELECT id, AI.SCORE(PROMPT('Is the review positive? {0}', body)) AS s,
               AI.CLASSIFY(body, ['praise', 'complaint', 'neutral remark']) AS kind
        FROM reviews
        WHERE AI.IF(PROMPT('Does the review discuss the ending? {0}', body))
        ORDER BY id
    """
    res = session.sql(q).run()
    t = res.table
    assert t.column_names == ["id", "s", "kind"]
    scores = t.column("s").to_pylist()
    assert all(0.0 <= s <= 1.0 for s in scores)
    assert set(t.column("kind").to_pylist()) <= {"praise", "complaint", "neutral remark"}
    kept = session.sql("SELECT id FROM reviews WHERE AI.IF(PROMPT('Does the review discuss the ending? {0}', body))"
                       ).collect().column("id").to_pylist()
    assert t.column("id").to_pylist() == sorted(kept)


def test_classify_label_scores_match_teacher_forcing(session):
    """A multi-token label's score is the sum of its tokens' log-probabilities."""
    import torch
    from quail_b200.api.prompts import bind_classify_prompt
    eng = session.engine()
    labels = ["praise", "complaint"]
    bp = bind_classify_prompt(None, labels)
    doc = "great story and a bad ending"
    out = eng.run_region(bp.preamble, [doc], [CallSpec(kind="classify", tail=bp.tail, name="c", labels=labels,
                                                       probabilities=True)])
    tok = eng.tokenizer
    ctx = np.concatenate([tok.encode(bp.preamble), tok.encode(doc), tok.encode(bp.tail)])
    model = eng.model
    scores = []
    for lab in labels:
        ids = tok.encode(lab)
        total = 0.0
        for j in range(len(ids)):
            seq = np.concatenate([ctx, ids[:j]])
            logits = _full_logits(model, seq)
            total += float(torch.log_softmax(logits, -1)[ids[j]])
        scores.append(total)
    probs = out.values[0]["c#probs"]
    want = torch.softmax(torch.tensor(scores), 0).tolist()
    assert np.allclose(probs, want, atol=1e-3)
    assert out.values[0]["c"] == labels[int(np.argmax(scores))]


def _full_logits(model, tokens):
    import torch
    from quail_b200.ops import reference as ref
    cfg = model.cfg
    T = len(tokens)
    h = model.embed[torch.as_tensor(tokens).long()]
    pos = torch.arange(T)
    QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
    for L in model.layers:
        x = ref.rmsnorm(h, L["ln1"], cfg.rms_eps)
        q = ref.rope_neox(ref.rmsnorm((x @ L["wq"].t()).view(T, QH, D), L["qn"], cfg.rms_eps), pos, model.cos_sin)
        k = ref.rope_neox(ref.rmsnorm((x @ L["wk"].t()).view(T, KH, D), L["kn"], cfg.rms_eps), pos, model.cos_sin)
        v = (x @ L["wv"].t()).view(T, KH, D)
        k, v = k.repeat_interleave(QH // KH, 1), v.repeat_interleave(QH // KH, 1)
        o = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                                             is_causal=True, scale=model.scale)
        h = h + o.transpose(0, 1).reshape(T, -1) @ L["wo"].t()
        x = ref.rmsnorm(h, L["ln2"], cfg.rms_eps)
        h = h + ref.silu_mul(x @ L["wg"].t(), x @ L["wu"].t()) @ L["wd"].t()
    return (ref.rmsnorm(h[-1:], model.final_norm, cfg.rms_eps) @ model.head.t())[0]


def test_map_greedy_decoding_matches_step_by_step_argmax(session):
    from quail_b200.api.prompts import bind_map_prompt
    eng = session.engine()
    bp = bind_map_prompt("Summarize the review in a few words.")
    doc = "too long and the ending made no sense"
    out = eng.run_region(bp.preamble, [doc], [CallSpec(kind="map", tail=bp.tail, name="m", max_tokens=5)])
    tok = eng.tokenizer
    seq = list(np.concatenate([tok.encode(bp.preamble), tok.encode(doc), tok.encode(bp.tail)]))
    gen = []
    for _ in range(5):
        nxt = int(_full_logits(eng.model, np.asarray(seq)).argmax())
        if nxt in tok.eos_ids:
            break
        gen.append(nxt)
        seq.append(nxt)
    assert out.values[0]["m"] == tok.decode(gen)


def test_sql_relational_operators(session):
    t = session.sql("SELECT grp, COUNT(*) AS n, MAX(id) AS top FROM reviews GROUP BY grp ORDER BY grp").collect()
    assert t.column("grp").to_pylist() == [0, 1, 2]
    assert t.column("n").to_pylist() == [8, 8, 8]
    t = session.sql("SELECT id, CASE WHEN id < 3 THEN 'low' ELSE 'high' END AS band FROM reviews "
                    "WHERE id IN (1, 2, 5) ORDER BY id DESC LIMIT 2").collect()
    assert t.to_pydict() == {"id": [5, 2], "band": ["high", "low"]}
    t = session.sql("WITH small AS (SELECT id FROM reviews WHERE id < 4) SELECT COUNT(*) AS n FROM small").collect()
    assert t.column("n").to_pylist() == [4]


def test_join_then_ai(session):
    aspects = pa.table({"aid": [0, 1], "grp": [0, 2]})
    session.register("aspects", aspects)
    t = session.sql("SELECT r.id, a.aid FROM reviews r JOIN aspects a ON r.grp = a.grp "
                    "WHERE AI.IF(PROMPT('Is it short? {0}', r.body)) ORDER BY r.id").collect()
    assert set(t.column("aid").to_pylist()) <= {0, 1}


def test_explain_lists_the_model_nodes(session):
    text = session.sql("SELECT id, AI.SCORE(PROMPT('ok? {0}', body)) FROM reviews "
                       "WHERE grp = 0 AND AI.IF(PROMPT('Is it long? {0}', body)) LIMIT 3").explain()
    assert "AiFilter" in text and "AiScore" in text and "Limit" in text and "Filter" in text


def test_unknown_model_is_refused():
    with pytest.raises(quail.RefusalError):
        quail.Session(config=quail.EngineConfig(model="no-such-model", device="cpu"))


def test_results_do_not_depend_on_chunk_size():
    t = _table(12, seed=3)
    outs = []
    for chunk in (48, 4096):
        cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=chunk)
        with quail.Session(config=cfg) as s:
            s.register("t", t)
            outs.append(s.sql("SELECT id, AI.SCORE(PROMPT('Good? {0}', body)) AS s FROM t ORDER BY id").collect())
    assert np.allclose(outs[0].column("s").to_pylist(), outs[1].column("s").to_pylist(), atol=1e-5)


def test_parallel_refusals():
    import pytest as _pytest

    from quail_b200.api.config import EngineConfig, RefusalError, check_config
    assert check_config(EngineConfig(model="qwen3-tiny", device="cpu")).name == "qwen3-tiny"
    with _pytest.raises(RefusalError, match="tensor parallelism runs dense Qwen3"):
        check_config(EngineConfig(model="qwen3.5-tiny", device="cpu", parallel="tp"))
    with _pytest.raises(RefusalError, match="expert parallelism needs"):
        check_config(EngineConfig(model="qwen3-tiny", device="cpu", parallel="ep"))
    with _pytest.raises(RefusalError, match="run on GPUs"):
        check_config(EngineConfig(model="qwen3-moe-gpu-tiny", device="cpu", parallel="ep", gpus=2))
    with _pytest.raises(RefusalError, match="does not split over 4 GPUs"):
        check_config(EngineConfig(model="qwen3-tiny", device="b200", parallel="tp", gpus=4))
    with _pytest.raises(RefusalError, match="divide gpus"):
        check_config(EngineConfig(model="qwen3-32b-fp8", device="b200", parallel="tp", gpus=4, group_gpus=8))
    # a TP=8 copy of the 32B model, and two TP=4 copies, are accepted
    assert check_config(EngineConfig(model="qwen3-32b-fp8", device="b200", parallel="tp", gpus=8)).layers == 64
    assert check_config(EngineConfig(model="qwen3-32b-fp8", device="b200", parallel="tp", gpus=8, group_gpus=4))
    with _pytest.raises(RefusalError, match="parallel is"):
        check_config(EngineConfig(model="qwen3-tiny", device="cpu", parallel="pp"))


def _both_ways(session, q):
    on = session.sql(q).run()
    session.settings["quail.pushdown"] = "false"
    try:
        off = session.sql(q).run()
    finally:
        session.settings.pop("quail.pushdown")
    return on, off


def test_case_guard_on_the_model_asks_only_where_the_filter_holds(session):
    f = "AI.IF(PROMPT('Does the review discuss the ending? {0}', body))"
    sc = "AI.SCORE(PROMPT('Is the review positive? {0}', body))"
    q = f"SELECT id, {f} AS f, CASE WHEN {f} THEN {sc} END AS s FROM reviews ORDER BY id"
    on, off = _both_ways(session, q)
    assert on.table.column("f").to_pylist() == off.table.column("f").to_pylist()
    for keep, a, b in zip(on.table.column("f").to_pylist(), on.table.column("s").to_pylist(),
                          off.table.column("s").to_pylist()):
        if keep:
            assert abs(a - b) < 1e-4
        else:
            assert a is None and b is None
    assert on.report["asked"] < off.report["asked"]


def test_a_first_call_left_out_on_a_row_still_reads_the_document(session):
    # the guarded call comes first in the region: rows it skips prefill the document alone,
    # then the unguarded call reads it as a follow-up question
    s1 = "AI.SCORE(PROMPT('Is the review positive? {0}', body))"
    s2 = "AI.SCORE(PROMPT('Is the review about money? {0}', body))"
    q = f"SELECT id, CASE WHEN grp = 1 THEN {s1} END AS a, {s2} AS b FROM reviews ORDER BY id"
    on, off = _both_ways(session, q)
    ta, tb = on.table, off.table
    for g, a_on, a_off, b_on, b_off in zip(ta.column("id").to_pylist(), ta.column("a").to_pylist(),
                                           tb.column("a").to_pylist(), ta.column("b").to_pylist(),
                                           tb.column("b").to_pylist()):
        assert abs(b_on - b_off) < 1e-4
        if g % 3 == 1:
            assert abs(a_on - a_off) < 1e-4
        else:
            assert a_on is None
    assert on.report["asked"] < off.report["asked"]


def test_projection_calls_ride_in_the_filter_region(session):
    # the WHERE filter and the SELECT list's calls on the same document run as one region:
    # the document is prefilled once, and the score is asked only where the filter kept the row
    q = ("SELECT id, AI.SCORE(PROMPT('Is the review positive? {0}', body)) AS s FROM reviews "
         "WHERE AI.IF(PROMPT('Does the review discuss the ending? {0}', body)) ORDER BY id")
    res = session.sql(q).run()
    assert len(res.report["regions"]) == 1
    kept = res.table.num_rows
    assert res.report["asked"] == 24 + kept
    alone = session.sql("SELECT id FROM reviews WHERE AI.IF(PROMPT('Does the review discuss the ending? {0}', "
                        "body)) ORDER BY id").collect()
    assert res.table.column("id").to_pylist() == alone.column("id").to_pylist()


def test_calls_written_almost_the_same(session):
    from quail_b200.sql.similar import likeness
    assert likeness("Is {0} rude?", "is {0} rude") == "spelling"
    assert likeness("Is the review about the ending? {0}", "Is the reveiw about the ending? {0}") == "typo"
    assert likeness("Is it from 2027? {0}", "Is it from 2028? {0}") is None
    assert likeness("Is {0} long?", "Is {0} short?") is None
    with pytest.raises(Exception, match="case, whitespace or punctuation"):
        session.sql("SELECT id FROM reviews WHERE AI.IF(PROMPT('Is {0} rude?', body)) "
                    "AND AI.IF(PROMPT('is {0} rude', body))").collect()
    res = session.sql("SELECT id, AI.SCORE(PROMPT('Is the review about the ending? {0}', body)) AS a, "
                      "AI.SCORE(PROMPT('Is the reveiw about the ending? {0}', body)) AS b FROM reviews").run()
    assert any("a few letters" in w for w in res.report["warnings"])
