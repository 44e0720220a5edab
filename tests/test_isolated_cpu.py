"""Document-isolated models (mammoth-1 / elephant-1) on the CPU engine.

The reference's "document_isolated" mask (quail/backends/quail/executor/
attention.py:371-375, quail/specs/base.py:174-181): the system turn and the
document form one block whose tokens read each other both ways; each question
reads that block and itself, whole. Answers are the LM head's logits of the
option letters at the prompt's last row (the slot_lm readout, readout.py:558).
The dense stand-in's answers are checked against a Hugging Face Qwen3 forward
over the whole prompt with that mask written out as a 4-D additive mask.
"""

import math

import numpy as np
import pyarrow as pa
import pytest
import torch

import quail_b200 as quail
from quail_b200.api import prompts as P
from quail_b200.api.config import EngineConfig
from quail_b200.api.engine import CallSpec, ModelEngine
from quail_b200.models.config import MODEL_CONFIGS
from quail_b200.ops import reference as ref

DOCS = ["the invoice was paid in full on the first of march",
        "a short note",
        "shipping delayed by weather; the customer asked for a refund and the order was cancelled " * 3]


def test_reference_attention_reads_a_flagged_own_segment_both_ways():
    g = torch.Generator().manual_seed(0)
    P_, KH, QH, D = 16, 2, 4, 32
    kc = torch.randn(8, P_, KH, D, generator=g)
    vc = torch.randn(8, P_, KH, D, generator=g)
    q = torch.randn(20, QH, D, generator=g)
    # one sequence: a 12-token resident block, then 20 own tokens
    seqs = torch.tensor([[0, 20, 2, 1, 12, 20, 0, 0, 0, 1, 0, 0]], dtype=torch.int32)
    pl = torch.tensor([3, 5, 1, 7], dtype=torch.int32)
    out = ref.segmented_attention(q, kc, vc, seqs, pl, 0.2)
    k_all = torch.cat([kc.view(-1, KH, D)[pl[0] * P_:pl[0] * P_ + 12],
                       torch.cat([kc[pl[1]], kc[pl[2]]])[:20]])
    v_all = torch.cat([vc.view(-1, KH, D)[pl[0] * P_:pl[0] * P_ + 12],
                       torch.cat([vc[pl[1]], vc[pl[2]]])[:20]])
    kr = k_all.repeat_interleave(QH // KH, dim=1)
    vr = v_all.repeat_interleave(QH // KH, dim=1)
    s = torch.einsum("thd,khd->htk", q, kr) * 0.2
    want = torch.einsum("htk,khd->thd", s.softmax(-1), vr)
    assert torch.allclose(out.view(20, QH, D), want, atol=1e-5)
    causal = seqs.clone()
    causal[0, 3] = 0
    assert not torch.allclose(ref.segmented_attention(q, kc, vc, causal, pl, 0.2).view(20, QH, D), want, atol=1e-3)


def _hf_model(cfg, ckpt):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    hc = Qwen3Config(vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                     num_hidden_layers=cfg.layers, num_attention_heads=cfg.num_q_heads,
                     num_key_value_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_eps,
                     rope_theta=cfg.rope_theta, tie_word_embeddings=cfg.tied_head,
                     max_position_embeddings=cfg.max_position)
    m = Qwen3ForCausalLM(hc).eval()
    m.config._attn_implementation = "eager"
    missing, _ = m.load_state_dict({k: v.float() for k, v in ckpt.items()}, strict=False)
    assert not [k for k in missing if "rotary" not in k], missing
    return m


def _letter_logits(hf, block, question, letters, isolated=True):
    ids = torch.as_tensor(np.concatenate([block, question]), dtype=torch.long)[None]
    T, B = ids.shape[1], len(block)
    allow = torch.tril(torch.ones(T, T, dtype=torch.bool))
    if isolated:
        allow[:B, :B] = True        # the block reads itself both ways
        allow[B:, :] = True         # each question reads the block and itself, whole
    mask = torch.zeros(1, 1, T, T)
    mask[0, 0][~allow] = float("-inf")
    with torch.no_grad():
        logits = hf(input_ids=ids, attention_mask=mask).logits[0, -1]
    return [float(logits[i]) for i in letters]


@pytest.fixture(scope="module")
def dense():
    eng = ModelEngine(EngineConfig(model="isolated-dense-tiny", device="cpu"))
    from quail_b200.models.weights import random_checkpoint
    ckpt = random_checkpoint(eng.cfg, seed=0, dtype=torch.float32)
    return eng, _hf_model(eng.cfg, ckpt)


def test_scores_match_a_full_forward_with_the_isolated_mask(dense):
    eng, hf = dense
    tok = eng.tokenizer
    bp = P.bind_mammoth_prompt("Is {0} about a payment?", "score", P.prompt_model(eng.cfg).turn)
    assert bp.preamble.startswith("<|im_start|>system\nApply the question to the state.")
    assert bp.preamble.endswith("<state>\n") and bp.tail.endswith("Answer with one letter: A, B.")
    out = eng.run_region(bp.preamble, DOCS, [CallSpec(kind="score", tail=bp.tail, name="s", letters=bp.letters)])
    a, b = int(tok.encode("A")[0]), int(tok.encode("B")[0])
    close = tok.encode(P.MAMMOTH_DOCUMENT_CLOSE)
    question = tok.encode(bp.tail)
    differs = 0
    for doc, vals in zip(DOCS, out.values):
        block = np.concatenate([tok.encode(bp.preamble), tok.encode(doc), close])
        la, lb = _letter_logits(hf, block, question, [a, b])
        assert vals["s"] == pytest.approx(1.0 / (1.0 + math.exp(-(la - lb))), abs=2e-4)
        ca, cb = _letter_logits(hf, block, question, [a, b], isolated=False)
        differs += abs((la - lb) - (ca - cb)) > 1e-3
    assert differs == len(DOCS)          # a causal read of the same prompt answers otherwise
    # no shared prefix task: every document's block is prefilled with the system turn, and the
    # question is a follow-up reading it
    blocks = sum(len(tok.encode(bp.preamble)) + len(tok.encode(d)) + len(close) for d in DOCS)
    assert out.stats["fresh_tokens"] == blocks + len(DOCS) * len(question)


def test_classify_is_the_best_option_letter(dense):
    eng, hf = dense
    tok = eng.tokenizer
    labels = ["billing", "shipping", "other"]
    bp = P.bind_mammoth_choice_prompt("What is {0} about?", labels, ["", "delivery issues", ""],
                                      turn=P.prompt_model(eng.cfg).turn)
    assert "\n\nOptions:\nA. billing\nB. shipping: delivery issues\nC. other" in bp.tail
    assert bp.tail.endswith("\n\nAnswer with one letter: A, B, C.") and bp.letters == ["A", "B", "C"]
    out = eng.run_region(bp.preamble, DOCS, [CallSpec(kind="classify", tail=bp.tail, name="c", labels=labels,
                                                      letters=bp.letters, probabilities=True)])
    ids = [int(tok.encode(x)[0]) for x in bp.letters]
    close = tok.encode(P.MAMMOTH_DOCUMENT_CLOSE)
    for doc, vals in zip(DOCS, out.values):
        block = np.concatenate([tok.encode(bp.preamble), tok.encode(doc), close])
        got = _letter_logits(hf, block, tok.encode(bp.tail), ids)
        assert vals["c"] == labels[int(np.argmax(got))]
        e = np.exp(np.asarray(got) - max(got))
        assert vals["c#probs"] == pytest.approx(list(e / e.sum()), abs=1e-4)


def test_two_calls_share_one_block(dense):
    eng, _ = dense
    turn = P.prompt_model(eng.cfg).turn
    f = P.bind_mammoth_prompt("Is {0} about a refund?", "filter", turn)
    s = P.bind_mammoth_prompt("Is {0} urgent?", "score", turn)
    both = eng.run_region(f.preamble, DOCS, [CallSpec(kind="filter", tail=f.tail, name="f", letters=f.letters,
                                                      drops=False),
                                             CallSpec(kind="score", tail=s.tail, name="s", letters=s.letters)])
    alone = eng.run_region(s.preamble, DOCS, [CallSpec(kind="score", tail=s.tail, name="s", letters=s.letters)])
    for x, y in zip(both.values, alone.values):
        assert x["s"] == pytest.approx(y["s"], abs=1e-5)   # the question reads only its block
    assert both.stats["asked"] == 2 * len(DOCS)


def test_sql_session_on_the_hybrid_stand_in():
    # Qwen3.5 layers (Gated DeltaNet stays causal, full attention reads the block both ways)
    with quail.Session(config=EngineConfig(model="mammoth-tiny", device="cpu")) as sess:
        t = pa.table({"id": list(range(len(DOCS))), "body": DOCS})
        sess.register("notes", quail.DocumentProvider.from_table(t, id_col="id"))
        out = sess.sql("SELECT id, AI.CLASSIFY(body, ['billing', 'shipping']) AS kind, "
                       "AI.SCORE(PROMPT('Is {0} urgent?', body)) AS urgency FROM notes "
                       "WHERE AI.IF(PROMPT('Is {0} written in English?', body))").collect()
        assert out.num_rows <= len(DOCS)
        assert set(out.column("kind").to_pylist()) <= {"billing", "shipping"}
        assert all(0.0 <= u <= 1.0 for u in out.column("urgency").to_pylist())
        # a generative-only function is refused with a reason
        with pytest.raises(Exception, match="decodes"):
            sess.sql("SELECT AI.MAP(body, 'summarize') FROM notes").collect()


def test_the_document_isolated_specs():
    for name in ("mammoth-1-bf16", "elephant-1-bf16"):
        cfg = MODEL_CONFIGS[name]
        assert cfg.bidirectional and cfg.readout == "slot_lm" and not cfg.decision_head
        assert cfg.is_hybrid and cfg.weight_dtype == "bf16" and not cfg.tied_head
    assert P.code_candidates(28)[-3:] == ["Z", "AA", "AB"]
    bp = P.bind_mammoth_choice_prompt(None, [f"l{i}" for i in range(30)])
    assert bp.tail.endswith("Answer with one label: " + ", ".join(P.code_candidates(30)) + ".")
    assert bp.tail.startswith("Question: Which option applies to the state?\n\nOptions:\nA. l0")
