"""DiffusionGemma's fp32 statement against Hugging Face's Gemma 4 text model, and its chunks.

The statement (quail_b200/models/gemma4.py) runs packed chunks over paged KV:
its logits must equal Hugging Face's Gemma4ForCausalLM on the same random
checkpoint (sliding and global layers, values from the key projection, a
quarter of the global frequency pairs rotated, GeGLU MLP beside the routed
experts, layer scalars, soft-capped tied head). Prompts packed with a shared
prefix, split across chunks, must match the same prompts alone, and a
sliding layer's window must reach into the earlier segments.
Reference: tests/gpu/test_diffusion_gemma_forward.py (forward against the
checkpoint's own implementation) and tests/engine/test_diffusion_gemma.py.
"""

import numpy as np
import pytest
import torch

from quail_b200.engine.arena import KVArena
from quail_b200.engine.stage_executor import StageExecutor, Task
from quail_b200.models import gemma4 as G
from quail_b200.models.config import MODEL_CONFIGS

CFG = MODEL_CONFIGS["diffusion-gemma-tiny"]


@pytest.fixture(scope="module")
def model():
    ckpt = G.random_gemma4(CFG, seed=3, dtype=torch.float32)
    ids = list(range(16))
    return ckpt, G.DiffusionGemmaReference(CFG, ckpt, head_rows=ids)


def _hf(ckpt):
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM
    m = Gemma4ForCausalLM(G.hf_config(CFG)).float().eval()
    sd = {k: v.float() for k, v in ckpt.items() if k != G.SELF_CONDITIONING_NORM}
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected and all(k == "lm_head.weight" for k in missing)
    m.tie_weights()
    return m


def _arena(pages=256, page=16):
    return KVArena.for_model(CFG, pages, page, device="cpu", dtype=torch.float32)


def _alone(model, tokens, full=False):
    arena = _arena()
    ex = StageExecutor(model, arena, 4096)
    got = {}
    ex.submit(Task(key="x", tokens=np.asarray(tokens, dtype=np.int32), pos_start=0, readout=True,
                   full_readout=full, on_done=lambda t, row: got.__setitem__("x", row.float())))
    ex.run()
    return got["x"]


def test_the_arena_keeps_each_layer_geometry():
    a = _arena(8)
    assert a.layer(0)[0].shape[-2:] == (CFG.num_kv_heads, CFG.head_dim)
    assert a.layer(1)[0].shape[-2:] == (CFG.full_kv_heads, CFG.full_head_dim)
    assert a.layer(2)[0].data_ptr() != a.layer(0)[0].data_ptr()


@pytest.mark.parametrize("n", [12, 40])
def test_statement_matches_hugging_face(model, n):
    ckpt, m = model
    hf = _hf(ckpt)
    rng = np.random.default_rng(n)
    toks = rng.integers(0, 4000, n)
    with torch.no_grad():
        logits = hf(torch.as_tensor(toks)[None]).logits[0, -1].float()
    row = _alone(m, toks, full=True)
    want = logits[:16]
    assert torch.allclose(row[:16], want, rtol=1e-4, atol=1e-4), (row[:16] - want).abs().max()
    assert int(row[16]) == int(logits.argmax())                    # the full-vocabulary argmax
    assert float(row[17]) == pytest.approx(float(torch.logsumexp(logits, 0)), rel=1e-5)


@pytest.mark.parametrize("chunk_tokens", [24, 1000])
def test_packed_chunks_match_prompts_alone(model, chunk_tokens):
    _, m = model
    rng = np.random.default_rng(1)
    prefix = rng.integers(0, 1000, 20).astype(np.int32)
    docs = [rng.integers(0, 1000, k).astype(np.int32) for k in (3, 30, 9)]
    suffix = np.concatenate([rng.integers(0, 1000, 5), G.canvas_ids(CFG)]).astype(np.int32)
    arena = _arena()
    ex = StageExecutor(m, arena, chunk_tokens, min_piece=8)
    got = {}
    ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
    for i, d in enumerate(docs):
        ex.submit(Task(key=("d", i), tokens=np.concatenate([d, suffix]), pos_start=len(prefix),
                       reads=[("p", len(prefix))], readout=True,
                       on_done=lambda t, row, i=i: got.__setitem__(i, row.float())))
    ex.run()
    for i, d in enumerate(docs):
        want = _alone(m, np.concatenate([prefix, d, suffix]))
        assert torch.allclose(got[i], want, rtol=1e-4, atol=1e-4), (i, (got[i] - want).abs().max())
    ex.free("p")
    assert arena.pool.free_pages == arena.pool.num_pages


def test_canvas_rows_read_their_embedding_through_the_canvas_norm(model):
    _, m = model
    ids = G.canvas_ids(CFG)
    assert ids.shape == (CFG.canvas_tokens,) and (ids >= G.CANVAS_TOKEN_BASE).all()
    assert (G.canvas_ids(CFG) == ids).all()                       # the same after every question
    tok = torch.as_tensor(np.concatenate([[7], ids]))
    h = G.embed_rows(tok, m.embed, CFG.embed_scale, m.canvas_norm, CFG.rms_eps)
    plain = m.embed[int(ids[0]) - G.CANVAS_TOKEN_BASE] * CFG.embed_scale
    assert torch.allclose(h[1], G.rms(plain[None], m.canvas_norm, CFG.rms_eps)[0])
    assert torch.allclose(h[0], m.embed[7] * CFG.embed_scale)


def test_sliding_window_reaches_into_earlier_segments():
    """A sliding layer's window counts positions across the prefix and document segments."""
    from quail_b200.ops import reference as ref
    torch.manual_seed(0)
    P, KH, D, W = 4, 1, 8, 5
    k = torch.randn(16, P, KH, D)
    v = torch.randn(16, P, KH, D)
    q = torch.randn(3, 1, D)
    # two segments: 6 keys on pages 0-1, then an own segment of 3 on pages 2
    seqs = torch.tensor([[0, 3, 2, 0, 6, 3, 0, 0, 0, 2, 0, 0]], dtype=torch.int32)
    pl = torch.tensor([0, 1, 2], dtype=torch.int32)
    got = ref.segmented_attention(q, k, v, G.window_seqs(seqs, W), pl, 1.0)
    keys = torch.cat([k.reshape(-1, KH, D)[:6], k.reshape(-1, KH, D)[8:11]])[:, 0]
    vals = torch.cat([v.reshape(-1, KH, D)[:6], v.reshape(-1, KH, D)[8:11]])[:, 0]
    for t in range(3):
        pos = 6 + t
        lo = pos - W + 1
        s = q[t, 0] @ keys[lo:pos + 1].t()
        want = torch.softmax(s, 0) @ vals[lo:pos + 1]
        assert torch.allclose(got[t], want, atol=1e-5)


DOCS = ["the plot was thin", "a great cast and music", "the ending surprised me", "long and slow"]


@pytest.fixture(scope="module")
def engine():
    from quail_b200.api.config import EngineConfig
    from quail_b200.api.engine import ModelEngine
    return ModelEngine(EngineConfig(model="diffusion-gemma-tiny", device="cpu", chunk_tokens=256))


def _canvas_logits(eng, bp, doc, ids):
    """The statement's logits of `ids` at the canvas row of the whole prompt, asked alone."""
    tok = eng.tokenizer
    toks = np.concatenate([tok.encode(bp.preamble), tok.encode(doc), tok.encode(bp.tail), G.canvas_ids(CFG)])
    eng.model.set_answer_rows(ids)
    return _alone(eng.model, toks)


def test_scores_are_read_at_the_canvas_row(engine):
    from quail_b200.api import prompts as P
    from quail_b200.api.engine import CallSpec
    tok = engine.tokenizer
    bp = P.bind_prompt("Is {0} about a film?", 1, P.prompt_model(CFG).turn)
    assert bp.preamble.startswith("<bos><|turn>system\n") and bp.tail.endswith("<channel|>")
    out = engine.run_region(bp.preamble, DOCS, [CallSpec(kind="score", tail=bp.tail, name="s")])
    t_ids, f_ids = tok.answer_ids(P.TRUE_SPELLINGS), tok.answer_ids(P.FALSE_SPELLINGS)
    both = set(t_ids) & set(f_ids)
    t_ids = [i for i in t_ids if i not in both]
    f_ids = [i for i in f_ids if i not in both]
    for doc, v in zip(DOCS, out.values):
        row = _canvas_logits(engine, bp, doc, t_ids + f_ids)
        margin = float(row[:len(t_ids)].max() - row[len(t_ids):].max())
        assert v["s"] == pytest.approx(1.0 / (1.0 + np.exp(-margin)), abs=1e-4)


def _hf_canvas_probs(hf, m, prompt, canvas, letter_ids):
    """Hugging Face's Gemma 4 on prompt + answer canvas: the prompt causal, the canvas rows
    reading the whole prompt (sliding layers: within the window) and each other both ways;
    canvas rows embedded through the canvas norm. Softmax of the letters at canvas row 0."""
    ids = torch.as_tensor(np.concatenate([prompt, canvas]).astype(np.int64))
    n, L = len(prompt), len(prompt) + len(canvas)
    emb = G.embed_rows(ids, m.embed, CFG.embed_scale, m.canvas_norm, CFG.rms_eps)[None]
    i = torch.arange(L)[:, None]
    j = torch.arange(L)[None, :]
    see = (j <= i) | ((i >= n) & (j >= n))
    slide = see & ((j > i - CFG.sliding_window) | ((i >= n) & (j >= n)))
    neg = torch.finfo(torch.float32).min

    def mask(ok):
        return torch.where(ok, 0.0, neg)[None, None].float()
    with torch.no_grad():
        logits = hf(inputs_embeds=emb, attention_mask={"full_attention": mask(see),
                                                       "sliding_attention": mask(slide)}).logits[0, n].float()
    return torch.softmax(logits[letter_ids], 0).numpy()


def test_classify_reads_row_zero_of_the_answer_canvas(engine):
    """Letters at row 0 of a 16-row answer canvas read both ways, against Hugging Face's model
    with that mask; an uncertain first draw is averaged over the further draws."""
    from quail_b200.api import prompts as P
    from quail_b200.api.engine import CallSpec
    ckpt = G.random_gemma4(CFG, seed=engine.config.seed, dtype=torch.float32)
    hf = _hf(ckpt)
    hf.config._attn_implementation = "eager"
    labels = ["praise", "complaint", "question"]
    bp = P.bind_letters_classify_prompt(None, labels, turn=P.prompt_model(CFG).turn)
    assert bp.letters == ["A", "B", "C"] and "- B: complaint" in bp.tail
    out = engine.run_region(bp.preamble, DOCS, [CallSpec(kind="classify", tail=bp.tail, name="k", labels=labels,
                                                         letters=bp.letters, probabilities=True)])
    tok = engine.tokenizer
    ids = [int(tok.encode(x)[0]) for x in bp.letters]
    draws = engine.config.canvas_draws
    for r, (doc, v) in enumerate(zip(DOCS, out.values)):
        prompt = np.concatenate([tok.encode(bp.preamble), tok.encode(doc), tok.encode(bp.tail)])
        first = _hf_canvas_probs(hf, engine.model, prompt, G.answer_canvas(CFG, r, 0), ids)
        entropy = float(-(first * np.log(first)).sum())
        ps = [first] if entropy <= G.CANVAS_ENTROPY_NATS else [first] + [
            _hf_canvas_probs(hf, engine.model, prompt, G.answer_canvas(CFG, r, d), ids) for d in range(1, draws)]
        mean = np.mean(ps, axis=0)
        assert v["k"] == labels[int(np.argmax(mean))]
        assert np.allclose(v["k#probs"], mean, atol=1e-4), (v["k#probs"], mean)


def test_answer_canvas_rows():
    c0, c1 = G.answer_canvas(CFG, 3, 0), G.answer_canvas(CFG, 3, 1)
    assert len(c0) == CFG.canvas_answer_rows and (c0 >= G.CANVAS_TOKEN_BASE).all()
    assert c0[1] - G.CANVAS_TOKEN_BASE == CFG.canvas_turn_close and (c0[2:] - G.CANVAS_TOKEN_BASE == CFG.canvas_pad).all()
    assert (G.answer_canvas(CFG, 3, 0) == c0).all() and c0[0] != c1[0]     # seeded per document and draw


def test_sql_on_the_canvas_model():
    import pyarrow as pa

    import quail_b200 as quail
    from quail_b200.api.config import RefusalError
    cfg = quail.EngineConfig(model="diffusion-gemma-tiny", device="cpu", chunk_tokens=256)
    with quail.Session(config=cfg) as s:
        s.register("r", quail.DocumentProvider.from_table(pa.table({"id": [0, 1, 2], "body": DOCS[:3]}),
                                                          id_col="id"))
        rows = s.sql("SELECT id, AI.CLASSIFY(body, ['praise', 'complaint']) AS k, "
                     "AI.SCORE(PROMPT('Is {0} long?', body)) AS sc FROM r ORDER BY id").collect().to_pylist()
        assert [r["k"] in ("praise", "complaint") for r in rows] == [True] * 3
        assert all(0.0 < r["sc"] < 1.0 for r in rows)
        for q in ("SELECT AI.MAP(body, 'Summarize.') FROM r",
                  "SELECT AI.EXTRACT(body, {'who': 'Who?'}) FROM r"):
            with pytest.raises(RefusalError, match="one denoising step"):
                s.sql(q).collect()
