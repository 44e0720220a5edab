"""The arena, packer and stage executor on CPU with the fp32 model.

The check that matters: packing rows into chunks (shared prefix read through
its pages, documents split into prefill pieces, follow-up questions reading a
document's pages) gives the same readout logits as running every prompt alone
through the plain causal model.
"""

import numpy as np
import pytest
import torch

from quail_b200.engine.arena import KVArena, PagePool
from quail_b200.engine.region import Call, RegionRun
from quail_b200.engine.stage_executor import StageExecutor, Task
from quail_b200.models.config import QWEN3_TINY
from quail_b200.models.qwen3 import Qwen3Reference
from quail_b200.models.weights import random_checkpoint
from quail_b200.ops import reference as ref


def _model(cfg=QWEN3_TINY, answer_ids=(11, 12, 13, 14)):
    ckpt = random_checkpoint(cfg.with_(vocab=1000, max_position=4096), seed=3, dtype=torch.float32)
    cfg = cfg.with_(vocab=1000, max_position=4096)
    return cfg, Qwen3Reference(cfg, ckpt, head_rows=answer_ids)


def _plain_logits(model, cfg, tokens):
    """Logits of the last token of one prompt, no arena, plain causal attention."""
    T = len(tokens)
    h = model.embed[torch.as_tensor(tokens).long()]
    pos = torch.arange(T)
    QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
    for L in model.layers:
        x = ref.rmsnorm(h, L["ln1"], cfg.rms_eps)
        q = ref.rope_neox(ref.rmsnorm((x @ L["wq"].t()).view(T, QH, D), L["qn"], cfg.rms_eps), pos, model.cos_sin)
        k = ref.rope_neox(ref.rmsnorm((x @ L["wk"].t()).view(T, KH, D), L["kn"], cfg.rms_eps), pos, model.cos_sin)
        v = (x @ L["wv"].t()).view(T, KH, D)
        k = k.repeat_interleave(QH // KH, 1)
        v = v.repeat_interleave(QH // KH, 1)
        o = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                                             is_causal=True, scale=model.scale)
        h = h + o.transpose(0, 1).reshape(T, -1) @ L["wo"].t()
        x = ref.rmsnorm(h, L["ln2"], cfg.rms_eps)
        h = h + ref.silu_mul(x @ L["wg"].t(), x @ L["wu"].t()) @ L["wd"].t()
    n = ref.rmsnorm(h[-1:], model.final_norm, cfg.rms_eps)
    return (n @ model.answer_rows.t())[0]


def test_page_pool_borrow_and_free():
    pool = PagePool(10, 4)
    assert pool.alloc("a", 9) == [0, 1, 2]
    assert pool.alloc("b", 4) == [3]
    pool.borrow("b", "a")
    pool.free_key("a")
    assert pool.free_pages == 6  # a's pages still held by b
    pool.check()
    pool.free_key("b")
    assert pool.free_pages == 10
    pool.check()
    assert pool.alloc("c", 41) is None


def test_retained_eviction():
    pool = PagePool(4, 4)
    pool.alloc("a", 8)
    pool.retain("a")
    pool.alloc("b", 4)
    pool.retain("b")
    assert pool.evict_retained(3) == ["a"]
    assert pool.free_pages == 3
    pool.check()


@pytest.mark.parametrize("chunk_tokens,page_tokens", [(64, 16), (1000, 128), (37, 8)])
def test_packed_chunks_match_plain_prompts(chunk_tokens, page_tokens):
    cfg, model = _model()
    arena = KVArena(cfg.layers, 64, page_tokens, cfg.num_kv_heads, cfg.head_dim, device="cpu",
                    dtype=torch.float32)
    ex = StageExecutor(model, arena, chunk_tokens, min_piece=4)
    rng = np.random.default_rng(0)
    prefix = rng.integers(0, 1000, 10).astype(np.int32)
    docs = [rng.integers(0, 1000, n).astype(np.int32) for n in (5, 40, 17, 90, 3)]
    suffix = rng.integers(0, 1000, 6).astype(np.int32)
    got = {}
    ex.submit(Task(key="prefix", tokens=prefix, pos_start=0, free_after=False))
    for i, d in enumerate(docs):
        toks = np.concatenate([d, suffix])
        ex.submit(Task(key=("d", i), tokens=toks, pos_start=len(prefix), reads=[("prefix", len(prefix))],
                       readout=True, on_done=lambda t, row, i=i: got.__setitem__(i, row.clone())))
    ex.run()
    ex.free("prefix")
    assert arena.pool.free_pages == arena.num_pages
    for i, d in enumerate(docs):
        want = _plain_logits(model, cfg, np.concatenate([prefix, d, suffix]))
        torch.testing.assert_close(got[i], want, rtol=1e-4, atol=1e-4)


def test_region_followup_questions_read_document_pages():
    cfg, model = _model()
    arena = KVArena(cfg.layers, 128, 16, cfg.num_kv_heads, cfg.head_dim, device="cpu", dtype=torch.float32)
    ex = StageExecutor(model, arena, 80, min_piece=4)
    rng = np.random.default_rng(1)
    prefix = rng.integers(0, 1000, 12).astype(np.int32)
    docs = [rng.integers(0, 1000, n).astype(np.int32) for n in (30, 7, 66)]
    s1 = rng.integers(0, 1000, 5).astype(np.int32)
    s2 = rng.integers(0, 1000, 9).astype(np.int32)
    calls = [Call(kind="score", suffix=s1, true_cols=[0, 1], false_cols=[2, 3], name="a"),
             Call(kind="score", suffix=s2, true_cols=[0], false_cols=[2], name="b")]
    res = RegionRun(ex, prefix, docs, calls).run()
    assert arena.pool.free_pages == arena.num_pages
    arena.pool.check()
    for r, d in enumerate(docs):
        la = _plain_logits(model, cfg, np.concatenate([prefix, d, s1]))
        lb = _plain_logits(model, cfg, np.concatenate([prefix, d, s2]))
        ma = max(la[0], la[1]) - max(la[2], la[3])
        mb = la.new_tensor(lb[0] - lb[2])
        assert abs(res[r].values["a"] - torch.sigmoid(ma).item()) < 1e-4
        assert abs(res[r].values["b"] - torch.sigmoid(mb).item()) < 1e-4


def test_filter_guards_followups():
    cfg, model = _model()
    arena = KVArena(cfg.layers, 128, 16, cfg.num_kv_heads, cfg.head_dim, device="cpu", dtype=torch.float32)
    ex = StageExecutor(model, arena, 200)
    rng = np.random.default_rng(2)
    prefix = rng.integers(0, 1000, 8).astype(np.int32)
    docs = [rng.integers(0, 1000, 20).astype(np.int32) for _ in range(12)]
    calls = [Call(kind="filter", suffix=rng.integers(0, 1000, 4).astype(np.int32), true_cols=[0], false_cols=[2],
                  name="f"),
             Call(kind="score", suffix=rng.integers(0, 1000, 4).astype(np.int32), true_cols=[1], false_cols=[3],
                  name="s")]
    res = RegionRun(ex, prefix, docs, calls).run()
    kept = [r for r in res if r.values["f"]]
    dropped = [r for r in res if not r.values["f"]]
    assert all("s" in r.values for r in kept)
    assert all("s" not in r.values for r in dropped)
    assert arena.pool.free_pages == arena.num_pages


class _CountingModel:
    """Full readouts whose argmax is the next token id: every row decodes to max_tokens."""

    def forward_chunk(self, chunk, arena):
        ids = torch.as_tensor(chunk.host["ids"]).long()
        rows = torch.as_tensor(chunk.host["final_rows"]).long()
        out = torch.zeros(rows.numel(), 4 + 2)
        out[:, 4] = ((ids[rows] + 1) % 500).float()
        return out


@pytest.mark.parametrize("pages", [64, 400])
def test_decode_headroom_under_memory_pressure(pages):
    """AI.MAP rows reserve their decode pages at admission, and decode steps are
    admitted before new documents, so a small arena finishes every row."""
    arena = KVArena(1, pages, 16, 1, 8, device="cpu", dtype=torch.float32)
    ex = StageExecutor(_CountingModel(), arena, 256)
    rng = np.random.default_rng(0)
    docs = [rng.integers(0, 500, int(n)).astype(np.int32) for n in rng.integers(20, 200, 40)]
    call = Call(kind="map", suffix=np.array([1, 2, 3], dtype=np.int32), max_tokens=24, stop_ids=(999,), name="m")
    res = RegionRun(ex, np.arange(48, dtype=np.int32), docs, [call], answer_width=4).run()
    for d, r in zip(docs, res):
        g = r.values["m"]
        assert len(g) == 24
        assert g[0] == (3 + 1) % 500 and g[1] == (g[0] + 1) % 500
    assert ex.pool.free_pages == pages
    ex.pool.check()


def test_copy_constrained_choice():
    """The copy state: the best candidate that continues a verbatim copy of the document wins,
    a stop token ends the phrase, and no qualifying candidate ends it too."""
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.ops.kernels import READOUT_TOPK as K

    class _Ex:
        pass
    doc = np.array([5, 6, 7, 5, 9], dtype=np.int32)
    call = Call(kind="extract", suffix=np.zeros(1, np.int32), stop_ids=(99,), copy=True, max_tokens=8)
    run = RegionRun(_Ex(), np.zeros(0, np.int32), [doc], [call], answer_width=2)

    def row(cands):
        c = list(cands) + [0] * (K - len(cands))
        return np.array([0.0, 0.0, 0.0, 0.0] + c + [0.0] * K, dtype=np.float32)   # 2 answers, arg, lse
    assert run._copy_choice(0, 0, row([3, 5]), 2, []) == 5          # 3 is not in the document
    assert run._copy_choice(0, 0, row([7, 6, 9]), 2, []) == 6       # after 5: 6 or 9 continue, 7 does not
    assert run._copy_choice(0, 0, row([5, 7]), 2, []) == 7          # after 5 6: only 7
    assert run._copy_choice(0, 0, row([1, 2]), 2, []) == 99         # nothing continues: the phrase ends
    run._copies.clear()
    assert run._copy_choice(0, 0, row([99, 5]), 2, []) == 99        # a stop token wins when ranked first


def test_extract_phrases_are_document_copies():
    """AI.EXTRACT on the fp32 model: every extracted phrase's tokens are a contiguous run of the
    row's document tokens (or empty)."""
    import pyarrow as pa

    import quail_b200 as quail
    from quail_b200.api import prompts as P
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=256)
    bodies = ["the order arrived late and the box was broken", "great service, thanks", "refund please"]
    with quail.Session(config=cfg) as s:
        s.register("t", pa.table({"id": [0, 1, 2], "body": bodies}))
        eng = s.engine()
        from quail_b200.engine.region import RegionRun
        seen = []
        orig = RegionRun._decode_step

        def spy(self, r, ci, row, generated):
            orig(self, r, ci, row, generated)
            seen.append((r, list(generated), self.docs[r].tolist()))
        RegionRun._decode_step = spy
        try:
            s.sql("SELECT id, AI.EXTRACT(body, ['What went wrong?']) AS e FROM t").collect()
        finally:
            RegionRun._decode_step = orig
        assert seen
        for r, gen, doc in seen:
            n = len(gen)
            assert n == 0 or any(doc[i:i + n] == gen for i in range(len(doc) - n + 1)), (gen, doc)
    del P, eng


def test_extract_drafts_match_token_by_token_decoding():
    """Document-copy drafts change how many passes an extraction takes, not what it extracts:
    the same region with drafts off gives the same phrases."""
    import pyarrow as pa

    import quail_b200 as quail
    from quail_b200.engine import region as R
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=256)
    bodies = ["the order arrived late and the box was broken", "great service, thanks a lot", "refund please now"]
    q = "SELECT id, AI.EXTRACT(body, ['What went wrong?', 'Who?']) AS e FROM t ORDER BY id"
    with quail.Session(config=cfg) as s:
        s.register("t", pa.table({"id": [0, 1, 2], "body": bodies}))
        with_drafts = s.sql(q).collect().column("e").to_pylist()
        keep = R.DRAFT_TOKENS
        R.DRAFT_TOKENS = 0
        try:
            without = s.sql(q).collect().column("e").to_pylist()
        finally:
            R.DRAFT_TOKENS = keep
    assert with_drafts == without


class _CopyModel:
    """A stand-in model that always predicts the current token + 1 (then a stop token): on a
    document of consecutive ids it copies the document, which exercises the drafts."""

    def __init__(self, stop):
        self.stop = stop

    def set_answer_rows(self, ids):
        pass

    def forward_chunk(self, chunk, arena):
        from quail_b200.ops.kernels import READOUT_TOPK as K
        ids = chunk.ids[chunk.final_rows.long()].float()
        R = ids.shape[0]
        out = torch.zeros(R, 1 + 2 + 2 * K)
        out[:, 1] = ids + 1                                   # argmax
        out[:, 3] = ids + 1                                   # top-1
        out[:, 4] = float(self.stop)                          # top-2: the stop token
        out[:, 3 + K] = 5.0
        out[:, 4 + K] = 4.0
        return out


@pytest.mark.parametrize("drafts", [0, 8])
def test_copy_drafts_accept_whole_runs(drafts):
    from quail_b200.engine import region as R
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.stage_executor import StageExecutor
    doc = np.arange(10, 31, dtype=np.int32)                   # 21 consecutive ids
    arena = KVArena(1, 64, 16, 1, 8, device="cpu", dtype=torch.float32)
    ex = StageExecutor(_CopyModel(stop=99), arena, 256)
    call = R.Call(kind="extract", suffix=np.array([9], dtype=np.int32), stop_ids=(99,), copy=True, max_tokens=30,
                  name="e")
    keep = R.DRAFT_TOKENS
    R.DRAFT_TOKENS = drafts
    try:
        run = R.RegionRun(ex, np.array([1, 2], dtype=np.int32), [doc], [call], answer_width=1)
        res = run.run()
    finally:
        R.DRAFT_TOKENS = keep
    assert res[0].values["e"] == list(range(10, 31))
    if drafts:
        assert run.drafted > 0 and ex.stats.passes <= 6
    else:
        assert run.drafted == 0 and ex.stats.passes >= 21


def test_extract_trace_lines(tmp_path, monkeypatch):
    """QUAIL_EXTRACT_TRACE writes one JSON line per copy-constrained choice."""
    import json

    from quail_b200.engine import region as R
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.stage_executor import StageExecutor
    path = tmp_path / "extract.jsonl"
    monkeypatch.setattr(R, "_EXTRACT_TRACE", str(path))
    doc = np.arange(10, 16, dtype=np.int32)
    arena = KVArena(1, 64, 16, 1, 8, device="cpu", dtype=torch.float32)
    ex = StageExecutor(_CopyModel(stop=99), arena, 256)
    call = R.Call(kind="extract", suffix=np.array([9], dtype=np.int32), stop_ids=(99,), copy=True, max_tokens=30,
                  name="e")
    run = R.RegionRun(ex, np.array([1, 2], dtype=np.int32), [doc], [call], answer_width=1)
    assert run.run()[0].values["e"] == list(range(10, 16))
    recs = [json.loads(ln) for ln in path.read_text().splitlines()]
    assert recs[0]["step"] == 0 and recs[0]["chosen"] == 10 and recs[0]["positions"] == 1
    assert recs[-1]["chosen"] == 99


def _score_engine(pages=None, retention=True):
    import quail_b200 as quail
    from quail_b200.api.engine import ModelEngine
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=96,
                             extra={"retention": retention})
    return ModelEngine(cfg, pages=pages)


def _score(engine, question, docs):
    from quail_b200.api.engine import CallSpec
    from quail_b200.api.prompts import bind_prompt
    bp = bind_prompt(question + " {0}")
    out = engine.run_region(bp.preamble, docs, [CallSpec(kind="score", tail=bp.tail, name="s")])
    return [v["s"] for v in out.values], out.stats


def _docs(n=14, seed=4):
    rng = np.random.default_rng(seed)
    words = ["alpha", "beta", "gamma", "delta", "omega", "kappa"]
    return [" ".join(rng.choice(words, size=int(rng.integers(10, 40)))) for _ in range(n)]


def test_retained_documents_are_read_again_without_a_prefill():
    docs = _docs()
    plain = _score_engine(retention=False)
    want1, _ = _score(plain, "Is it greek?", docs)
    want2, _ = _score(plain, "Is it long?", docs)
    eng = _score_engine()
    got1, st1 = _score(eng, "Is it greek?", docs)
    got2, st2 = _score(eng, "Is it long?", docs)
    assert st1["reused_documents"] == 0
    assert st2["reused_documents"] == len(docs) and st2["replays"] == 0
    assert st2["fresh_tokens"] < st1["fresh_tokens"]
    np.testing.assert_allclose(got1, want1, atol=1e-5)
    np.testing.assert_allclose(got2, want2, atol=1e-5)
    eng.arena.pool.check()


def test_evicted_documents_are_replayed_on_a_tiny_arena():
    docs = _docs(30, seed=5)
    plain = _score_engine(retention=False)
    want, _ = _score(plain, "Is it long?", docs)
    eng = _score_engine(pages=40)                   # far less than the 30 documents' pages
    _score(eng, "Is it greek?", docs)
    got, st = _score(eng, "Is it long?", docs)
    assert st["replays"] > 0 and st["reused_documents"] + st["replays"] == len(docs)
    np.testing.assert_allclose(got, want, atol=1e-5)
    eng.arena.pool.check()


def test_rewind_releases_a_first_decode_before_later_questions():
    from quail_b200.api.engine import CallSpec
    from quail_b200.api.prompts import bind_map_prompt, bind_prompt
    docs = _docs(8, seed=6)
    bm = bind_map_prompt("Name one word.")
    bs = bind_prompt("Is it greek? {0}")
    calls = [CallSpec(kind="map", tail=bm.tail, name="m", max_tokens=6), CallSpec(kind="score", tail=bs.tail, name="s")]
    eng = _score_engine(retention=False)
    out = eng.run_region(bm.preamble, docs, calls)
    # the same follow-up after a first question that generates nothing reads the same KV
    alone = _score_engine(retention=False)
    first = CallSpec(kind="score", tail=bm.tail, name="x")
    want_s = [v["s"] for v in alone.run_region(bm.preamble, docs, [first, calls[1]]).values]
    want_m = alone.run_region(bm.preamble, docs, calls[:1]).values
    np.testing.assert_allclose([v["s"] for v in out.values], want_s, atol=1e-5)
    assert [v["m"] for v in out.values] == [v["m"] for v in want_m]
    eng.arena.pool.check()
    assert not eng.arena.pool.owned                  # every key released at the end
