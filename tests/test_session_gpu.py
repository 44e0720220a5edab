"""The query API on a B200: SQL through the kernel pipeline (fp8 tiny Qwen3)."""

import numpy as np
import pyarrow as pa
import pytest

import quail_b200 as quail

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def session():
    rng = np.random.default_rng(0)
    words = ["ending", "music", "cast", "plot", "money", "great", "bad", "long"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 40)))) for _ in range(40)]
    cfg = quail.EngineConfig(model="qwen3-gpu-tiny", device="b200", chunk_tokens=2048)
    with quail.Session(config=cfg) as s:
        s.register("t", pa.table({"id": list(range(40)), "body": bodies}))
        yield s


def test_filter_is_the_projection_of_the_same_call(session):
    kept = session.sql("SELECT id FROM t WHERE AI.IF(PROMPT('Is it about music? {0}', body)) ORDER BY id").collect()
    flags = session.sql("SELECT id, AI.IF(PROMPT('Is it about music? {0}', body)) AS f FROM t ORDER BY id").collect()
    want = [i for i, f in zip(flags.column("id").to_pylist(), flags.column("f").to_pylist()) if f]
    assert kept.column("id").to_pylist() == want


def test_classify_map_and_score_on_the_kernels(session):
    t = session.sql("""
        SELECT id, AI.SCORE(PROMPT('Positive? {0}', body)) AS s,
               AI.CLASSIFY(body, ['praise', 'complaint'], {'probabilities': true}) AS k,
               AI.MAP(body, 'Summarize.', 4) AS m
        FROM t WHERE id < 6 ORDER BY id""").collect()
    assert t.num_rows == 6
    assert all(0.0 <= s <= 1.0 for s in t.column("s").to_pylist())
    assert set(t.column("k").to_pylist()) <= {"praise", "complaint"}
    assert all(isinstance(m, str) for m in t.column("m").to_pylist())



def test_decision_model_on_the_kernels():
    """A decision model (Qwen3 backbone on the bf16 kernels + option-scoring head) against
    the same weights in the fp32 reference model: same SQL, scores to bf16 accuracy."""
    import torch
    from quail_b200.api.engine import ModelEngine
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.build import random_checkpoint_on
    from quail_b200.models.qwen3 import Qwen3Reference
    rng = np.random.default_rng(1)
    words = ["refund", "late", "broken", "great", "thanks", "order"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 30)))) for _ in range(12)]
    q = ("SELECT id, AI.SCORE(PROMPT('Refund request? {0}', body)) AS s, "
         "AI.CLASSIFY(body, ['billing', 'shipping']) AS c FROM t ORDER BY id")
    cfg = quail.EngineConfig(model="decision-gpu-tiny", device="b200", chunk_tokens=2048)
    with quail.Session(config=cfg) as s:
        s.register("t", pa.table({"id": list(range(12)), "body": bodies}))
        got = s.sql(q).collect()
        eng = s.engine()
        m = eng.cfg
        ref_model = Qwen3Reference(m, random_checkpoint_on(m, eng.device, seed=0), device=eng.device)
        ref_model.decision = eng.model.decision
        arena = KVArena(m.layers, 4096, 16, m.num_kv_heads, m.head_dim, device=eng.device, dtype=torch.float32)
        s._engine = ModelEngine.from_replica(cfg, ref_model, arena, tokenizer=eng.tokenizer)
        want = s.sql(q).collect()
        s._engine = eng
    a, b = np.array(got.column("s").to_pylist()), np.array(want.column("s").to_pylist())
    assert np.all((a > 0) & (a < 1))
    # scores are sigmoid(yes - no); compare the logit differences, whose spread
    # over the 12 rows is what a wrong (constant, or shuffled) readout would lose
    da, db = np.log(a / (1 - a)), np.log(b / (1 - b))
    spread = db.max() - db.min()
    assert spread > 1e-3, f"the reference scores do not separate the rows: {db}"
    assert np.abs(da - db).max() < 0.2 * spread, (da, db)
    assert np.corrcoef(da, db)[0, 1] > 0.95, (da, db)
    agree = np.mean(np.array(got.column("c").to_pylist()) == np.array(want.column("c").to_pylist()))
    assert agree >= 0.9


def test_extract_copies_from_the_document(session):
    """AI.EXTRACT on the kernels with the copy constraint (top-k readout): every phrase is a
    verbatim piece of its row's document (or null when nothing was copied)."""
    t = session.sql("SELECT id, body, AI.EXTRACT(body, ['What is it about?']) AS e FROM t WHERE id < 12 "
                    "ORDER BY id").collect()
    for body, e in zip(t.column("body").to_pylist(), t.column("e").to_pylist()):
        for phrase in e:
            assert phrase is None or phrase.strip() in body, (phrase, body)


def test_reranker_model_on_the_kernels():
    """A Qwen3 reranker on the bf16 kernels against the same weights in the fp32 reference
    model: AI.SCORE = sigmoid(yes - no) of its chat prompt, to bf16 accuracy."""
    import torch
    from quail_b200.api.engine import ModelEngine
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.build import random_checkpoint_on
    from quail_b200.models.qwen3 import Qwen3Reference
    rng = np.random.default_rng(2)
    words = ["refund", "late", "broken", "great", "thanks", "order"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 30)))) for _ in range(12)]
    q = "SELECT id, AI.SCORE(PROMPT('Does {0} ask for a refund?', body)) AS s FROM t ORDER BY id"
    cfg = quail.EngineConfig(model="reranker-gpu-tiny", device="b200", chunk_tokens=2048)
    with quail.Session(config=cfg) as s:
        s.register("t", pa.table({"id": list(range(12)), "body": bodies}))
        got = s.sql(q).collect()
        eng = s.engine()
        m = eng.cfg
        ref_model = Qwen3Reference(m, random_checkpoint_on(m, eng.device, seed=0), device=eng.device)
        arena = KVArena(m.layers, 4096, 16, m.num_kv_heads, m.head_dim, device=eng.device, dtype=torch.float32)
        s._engine = ModelEngine.from_replica(cfg, ref_model, arena, tokenizer=eng.tokenizer)
        want = s.sql(q).collect()
        s._engine = eng
    a, b = np.array(got.column("s").to_pylist()), np.array(want.column("s").to_pylist())
    assert np.all((a > 0) & (a < 1))
    # scores are sigmoid(yes - no); compare the logit differences, whose spread
    # over the 12 rows is what a wrong (constant, or shuffled) readout would lose
    da, db = np.log(a / (1 - a)), np.log(b / (1 - b))
    spread = db.max() - db.min()
    assert spread > 1e-3, f"the reference scores do not separate the rows: {db}"
    assert np.abs(da - db).max() < 0.2 * spread, (da, db)
    assert np.corrcoef(da, db)[0, 1] > 0.95, (da, db)
