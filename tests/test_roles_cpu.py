"""Reranker and decision models end to end on CPU: prompts, refusals, head readouts.

Each answer is checked against the plain fp32 model run over the whole prompt
(no arena, no chunking): the decision head's scores of the option rows, the
reranker's yes-vs-no margin at the last row.
"""

import math

import numpy as np
import pyarrow as pa
import pytest
import torch

import quail_b200 as quail
from quail_b200.api import prompts as P
from quail_b200.api.config import RefusalError
from quail_b200.models.decision import DecisionHead, head_tensors, random_decision_head
from quail_b200.ops import reference as ref

from test_sae_cpu import _plain_hidden


def _table(n=9, seed=1):
    rng = np.random.default_rng(seed)
    words = ["refund", "late", "broken", "great", "thanks", "order", "never", "again", "fast", "box"]
    return pa.table({"id": list(range(n)),
                     "body": [" ".join(rng.choice(words, size=int(rng.integers(3, 14)))) for _ in range(n)]})


def _session(model):
    cfg = quail.EngineConfig(model=model, device="cpu", chunk_tokens=96)
    s = quail.Session(config=cfg)
    s.register("tickets", quail.DocumentProvider.from_table(_table(), id_col="id"))
    return s


@pytest.fixture(scope="module")
def decision():
    with _session("decision-tiny") as s:
        yield s


@pytest.fixture(scope="module")
def reranker():
    with _session("reranker-tiny") as s:
        yield s


def test_head_split_matches_one_statement():
    gen = torch.Generator().manual_seed(3)
    head = DecisionHead(head_tensors(random_decision_head(64, 16, gen)), "cpu")
    rows = torch.randn(5, 4, 64, generator=gen)          # 5 prompts: 3 options + the last row
    want = head.scores(rows[:, :3], rows[:, 3]).numpy()
    for p in range(5):
        got = head.combine(head.features(rows[p]).numpy())
        np.testing.assert_allclose(got, want[p], rtol=1e-5, atol=1e-5)


def test_head_tensor_checks():
    t = head_tensors(random_decision_head(8, 4, torch.Generator().manual_seed(0)))
    with pytest.raises(ValueError, match="missing"):
        head_tensors({"decision_head." + k: v for k, v in t.items() if k != "scalar.weight"})
    with pytest.raises(ValueError, match="does not use"):
        head_tensors({**{"decision_head." + k: v for k, v in t.items()}, "decision_head.extra": t["key.weight"]})


def test_decision2_prompt_text():
    bp = P.bind_decision_prompt("Is the customer asking for a refund? {0}", "filter")
    assert bp.preamble == "Context:\n"
    assert bp.segments == [
        "\n\nTask type: noul\nQuestion:\nIs the customer asking for a refund?\nOptions:",
        '\n<option>\n{"description":"No","key":"false"}\n</option>',
        '\n<option>\n{"description":"Yes","key":"true"}\n</option>',
        "\n\nSelect the single option best supported by the context and instructions.\nDecision:",
    ]
    assert bp.read == [1, 2] and bp.tail == "".join(bp.segments)
    cp = P.bind_decision_choice_prompt(None, ["billing", "shipping"], ["money matters", ""])
    assert cp.segments[0] == "\n\nTask type: choice\nQuestion:\n" + P.CHOICE_QUESTION + "\nOptions:"
    assert cp.segments[1] == '\n<option>\n{"description":"money matters","key":"billing"}\n</option>'
    assert cp.segments[2] == '\n<option>\n{"description":null,"key":"shipping"}\n</option>'
    assert cp.read == [1, 2]


def test_reranker_prompt_text():
    bp = P.bind_reranker_prompt("Does {0} mention a refund?")
    assert bp.question == "Does this document mention a refund?"
    assert bp.preamble.startswith("<|im_start|>system\nYou are an expert at text analysis. Judge whether")
    assert bp.preamble.endswith("<Query>: Does this document mention a refund?\n<Document>: ")
    assert bp.tail == "<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n"
    assert P.bind_reranker_prompt("{0} Is it about shipping?").question == "Is it about shipping?"


def _decision_scores(eng, bp, body):
    """Option scores of one row from the plain model over the whole prompt."""
    tok, model, cfg = eng.tokenizer, eng.model, eng.cfg
    parts = [tok.encode(s) for s in bp.segments]
    seq = np.concatenate([tok.encode(bp.preamble), tok.encode(body)] + parts)
    h = _plain_hidden(model, cfg, seq)
    ends, at = [], len(seq) - sum(len(p) for p in parts)
    for p in parts:
        at += len(p)
        ends.append(at - 1)
    rows = ref.rmsnorm(h[[ends[i] for i in bp.read] + [len(seq) - 1]], model.final_norm, cfg.rms_eps)
    return model.decision.scores(rows[None, :-1], rows[None, -1])[0].numpy()


def test_decision_filter_score_classify(decision):
    q = ("SELECT id, AI.SCORE(PROMPT('Is the customer asking for a refund? {0}', body)) AS s, "
         "AI.CLASSIFY(body, ['billing', 'shipping', 'praise']) AS c FROM tickets")
    t = decision.sql(q).collect()
    eng = decision.engine()
    bodies = _table().column("body").to_pylist()
    sp = P.bind_decision_prompt("Is the customer asking for a refund? {0}", "score")
    cp = P.bind_decision_choice_prompt(None, ["billing", "shipping", "praise"])
    for body, s, c in zip(bodies, t.column("s").to_pylist(), t.column("c").to_pylist()):
        sc = _decision_scores(eng, sp, body)
        assert s == pytest.approx(1 / (1 + math.exp(-(sc[1] - sc[0]))), rel=1e-4, abs=1e-5)
        cc = _decision_scores(eng, cp, body)
        assert c == ["billing", "shipping", "praise"][int(np.argmax(cc))]
    f = decision.sql("SELECT id FROM tickets WHERE AI.IF(PROMPT('Is the customer asking for a refund? {0}', body))"
                     ).collect()
    want = [i for i, s in enumerate(t.column("s").to_pylist()) if s > 0.5]
    assert sorted(f.column("id").to_pylist()) == want


def test_decision_refuses_text_output(decision):
    with pytest.raises(RefusalError, match="decodes the model's next tokens"):
        decision.sql("SELECT AI.MAP(body, 'Summarize.') FROM tickets").collect()


def test_reranker_score(reranker):
    t = reranker.sql("SELECT id, AI.SCORE(PROMPT('Does {0} mention a refund?', body)) AS s FROM tickets").collect()
    eng = reranker.engine()
    tok, model, cfg = eng.tokenizer, eng.model, eng.cfg
    bp = P.bind_reranker_prompt("Does {0} mention a refund?")
    yes, no = tok.answer_ids(["yes"])[0], tok.answer_ids(["no"])[0]
    head = model.head
    for body, s in zip(_table().column("body").to_pylist(), t.column("s").to_pylist()):
        seq = np.concatenate([tok.encode(bp.preamble), tok.encode(body), tok.encode(bp.tail)])
        h = ref.rmsnorm(_plain_hidden(model, cfg, seq)[-1:], model.final_norm, cfg.rms_eps)
        logits = (h @ head.t()).float()[0]
        m = float(logits[yes] - logits[no])
        assert s == pytest.approx(1 / (1 + math.exp(-m)), rel=1e-4, abs=1e-5)


def test_reranker_refusals(reranker):
    with pytest.raises(RefusalError, match="cannot run AI.CLASSIFY"):
        reranker.sql("SELECT AI.CLASSIFY(body, ['a', 'b']) FROM tickets").collect()
    with pytest.raises(RefusalError, match="only be used with AI.SCORE"):
        reranker.sql("SELECT id FROM tickets WHERE AI.IF(PROMPT('Is it late? {0}', body))").collect()
