"""AI.SAE_FEATURES end to end on CPU: SQL -> region -> SAE readout on the fp32 model."""

import numpy as np
import pyarrow as pa
import pytest
import torch

import quail_b200 as quail
from quail_b200.api.config import RefusalError
from quail_b200.api.prompts import bind_features_prompt
from quail_b200.engine.region import feature_list
from quail_b200.ops import reference as ref


def _table(n=10, seed=0):
    rng = np.random.default_rng(seed)
    words = ["ending", "music", "cast", "plot", "money", "great", "bad", "long", "short", "story"]
    return pa.table({"id": list(range(n)),
                     "body": [" ".join(rng.choice(words, size=int(rng.integers(3, 12)))) for _ in range(n)]})


@pytest.fixture(scope="module")
def session():
    cfg = quail.EngineConfig(model="qwen3-sae-tiny", device="cpu", chunk_tokens=256)
    with quail.Session(config=cfg) as s:
        s.register("reviews", quail.DocumentProvider.from_table(_table(), id_col="id"))
        yield s


def _plain_hidden(model, cfg, tokens):
    """Residual stream after the last layer for one prompt, plain causal attention, no arena."""
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
        o = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1),
                                                             v.transpose(0, 1), is_causal=True, scale=model.scale)
        h = h + o.transpose(0, 1).reshape(T, -1) @ L["wo"].t()
        x = ref.rmsnorm(h, L["ln2"], cfg.rms_eps)
        h = h + ref.silu_mul(x @ L["wg"].t(), x @ L["wu"].t()) @ L["wd"].t()
    return h


@pytest.mark.parametrize("pooling", ["last", "max"])
def test_sae_features_match_plain_model(session, pooling):
    tmpl = "{0} What is the review about?"
    q = f"SELECT id, AI.SAE_FEATURES(PROMPT('{tmpl}', body), {{'pooling': '{pooling}'}}) AS f FROM reviews"
    t = session.sql(q).collect()
    assert t.schema.field("f").type == pa.list_(pa.struct([("feature", pa.int32()), ("strength", pa.float32())]))
    eng = session.engine()
    model, cfg, tok = eng.model, eng.cfg, eng.tokenizer
    bp = bind_features_prompt(tmpl)
    pre = tok.encode(bp.preamble)
    for body, got in zip(_table().column("body").to_pylist(), t.column("f").to_pylist()):
        doc = tok.encode(body)
        own = np.concatenate([doc, tok.encode(bp.tail)])
        h = _plain_hidden(model, cfg, np.concatenate([pre, own]))
        rows = h[len(pre):] if pooling == "max" else h[-1:]
        want = feature_list(ref.sae_features(rows, model.sae_w, model.sae_b, cfg.sae_keep).numpy())
        got = [(d["feature"], d["strength"]) for d in got]
        assert [f for f, _ in got] == [f for f, _ in want]
        np.testing.assert_allclose([x for _, x in got], [x for _, x in want], rtol=1e-4, atol=1e-5)
        strengths = [x for _, x in got]
        assert strengths == sorted(strengths, reverse=True) and all(x > 0 for x in strengths)
        if pooling == "last":
            assert len(got) <= cfg.sae_keep


def test_feature_list_max_pools_rows():
    rows = np.array([[3, 1, 0, 2.0, 1.0, 0.0], [1, 5, 3, 4.0, 0.5, 1.5]], dtype=np.float32)
    assert feature_list(rows) == [(1, 4.0), (3, 2.0), (5, 0.5)]
    assert feature_list(rows[:1]) == [(3, 2.0), (1, 1.0)]


def test_sae_model_refuses_other_functions(session):
    with pytest.raises(RefusalError):
        session.sql("SELECT id FROM reviews WHERE AI.IF(PROMPT('Is it long? {0}', body))").collect()


def test_sae_needs_pooling_and_question(session):
    with pytest.raises(Exception):
        session.sql("SELECT AI.SAE_FEATURES(PROMPT('{0} What?', body)) FROM reviews").collect()
    with pytest.raises(Exception):
        session.sql("SELECT AI.SAE_FEATURES(PROMPT('About: {0}', body), {'pooling': 'last'}) FROM reviews").collect()
