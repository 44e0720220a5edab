"""Set attention (LiquidAI d1 / LFM3): pass layout, masks, pointer reads, and SQL on the CPU model.

Under set attention a pass is a document's state and up to the set size of
questions; the state reads every question of its pass and each question reads
the state and itself (quail/backends/quail/executor/models/lfm3.py:334-365,
set_passes.py). The CPU model is the fp32 statement with dense masks; its
pieces are checked against independent forms (a grouped conv1d for the short
convolution, the mask against the rule it states).
"""

import math

import numpy as np
import pyarrow as pa
import pytest
import torch
import torch.nn.functional as F

import quail_b200 as quail
from quail_b200.engine.set_passes import SetQuestion, SetRegion, pointer_span, split_passes
from quail_b200.models.config import MODEL_CONFIGS
from quail_b200.models.lfm3 import Lfm3Reference, SetPass, rotary_table, set_mask
from quail_b200.models.weights import random_checkpoint


def test_the_set_mask():
    p = SetPass(tokens=np.zeros(10, np.int32), state=4, questions=[3, 3])
    m = set_mask(p, "attn", 0)
    assert m[:4].all()                                   # the state reads its whole pass
    assert m[4:7, :7].all() and not m[4:7, 7:].any()     # question 1: the state and itself
    assert m[7:, :4].all() and m[7:, 7:].all() and not m[7:, 4:7].any()
    w = set_mask(p, "swa", 3)
    assert w[5, 3:6].all() and not w[5, :3].any() and not w[5, 6:].any()


def test_passes_split_by_set_size_and_budget():
    assert split_passes(10, [3, 3, 3, 3, 3], 2, set_size=2, budget=100) == [[0, 1], [2, 3], [4]]
    # state 10 + 5 + (2 + 5) = 22 fits; a third question (+7) does not fit 25
    assert split_passes(10, [5, 5, 5], 2, set_size=16, budget=25) == [[0, 1], [2]]
    with pytest.raises(ValueError, match="does not fit"):
        split_passes(20, [10], 2, set_size=4, budget=25)


def test_full_layers_rotate_half_the_frequency_pairs():
    cfg = MODEL_CONFIGS["d1-tiny"]
    full, swa = rotary_table(cfg, "attn"), rotary_table(cfg, "swa")
    half = cfg.head_dim // 2
    keep = int(cfg.rotary_pairs * half)
    assert torch.all(full[:, keep:half] == 1) and torch.all(full[:, half + keep:] == 0)
    assert torch.equal(full[:, :keep], swa[:, :keep])
    assert not torch.all(swa[30000, half + keep:] == 0)      # the sliding layers rotate every pair


def test_the_short_convolution_is_a_causal_grouped_conv():
    cfg = MODEL_CONFIGS["d1-tiny"]
    ckpt = random_checkpoint(cfg, seed=1, dtype=torch.float32)
    m = Lfm3Reference(cfg, ckpt)
    L = m.layers[0]
    x = torch.randn(9, cfg.hidden)
    got = m._conv(L, x)
    H, W = cfg.hidden, cfg.conv_width
    bcx = x @ L["win"].t()
    B, C, xx = bcx[:, :H], bcx[:, H:2 * H], bcx[:, 2 * H:]
    conv = F.conv1d((B * xx).t()[None], L["taps"][:, None, :], padding=W - 1, groups=H)[0, :, :9].t()
    assert torch.allclose(got, (C * conv) @ L["wout"].t(), atol=1e-4)


def test_pointer_reads():
    torch.manual_seed(0)
    H = 32
    doc = torch.randn(8, H)                  # row 0: nothing; rows 1..7: the document
    start, end = doc[3] * 6.0, doc[5] * 6.0  # point at document tokens 2..4
    first, last, found = pointer_span(start, end, doc, span_tokens=4)
    assert (first, last) == (3, 5) and found > 0.5
    first, last, found = pointer_span(doc[0] * 6.0, end, doc, span_tokens=4)
    assert (first, last) == (0, 0) and found < 0.5
    # the span cap: an end further than span_tokens rows from the start is not taken
    first, last, _ = pointer_span(doc[1] * 6.0, doc[7] * 6.0, doc, span_tokens=3)
    assert last - first < 3


def test_pass_mates_change_an_answer_through_the_state():
    cfg = MODEL_CONFIGS["d1-tiny"]
    m = Lfm3Reference(cfg, random_checkpoint(cfg, seed=2, dtype=torch.float32))
    rng = np.random.default_rng(0)
    state = rng.integers(0, cfg.vocab, 20).astype(np.int32)
    q1 = rng.integers(0, cfg.vocab, 6).astype(np.int32)
    q2 = rng.integers(0, cfg.vocab, 6).astype(np.int32)
    alone = m.forward_passes([SetPass(np.concatenate([state, q1]), 20, [6], [25])])[0]
    both = m.forward_passes([SetPass(np.concatenate([state, q1, q2]), 20, [6, 6], [25, 31])])[0]
    swapped = m.forward_passes([SetPass(np.concatenate([state, q2, q1]), 20, [6, 6], [25, 31])])[0]
    # the state read q2, so q1's answer row changes ...
    assert not torch.allclose(alone[0], both[0], atol=1e-4)
    # ... and where q1 sits in the pass matters only through positions and the sliding layers
    assert both.shape == swapped.shape == (2, cfg.hidden)


def test_region_answers_every_kind_in_shared_passes():
    cfg = MODEL_CONFIGS["d1-tiny"]
    m = Lfm3Reference(cfg, random_checkpoint(cfg, seed=3, dtype=torch.float32))
    rng = np.random.default_rng(1)
    head = np.arange(5, dtype=np.int32)
    header = np.asarray([7, 8], np.int32)
    docs = [rng.integers(10, 1000, n).astype(np.int32) for n in (12, 30, 7)]
    states = [np.concatenate([head, d, header]) for d in docs]
    spans = [(len(head), len(d)) for d in docs]
    qs = [SetQuestion("yes_no", rng.integers(10, 1000, 5).astype(np.int32), yes=[11], no=[12]),
          SetQuestion("score", rng.integers(10, 1000, 5).astype(np.int32), yes=[11], no=[12]),
          SetQuestion("choice", rng.integers(10, 1000, 6).astype(np.int32), options=[[21], [22], [23]]),
          SetQuestion("read", rng.integers(10, 1000, 6).astype(np.int32), slots=(2, 0))]
    region = SetRegion(m, m.head, chunk_tokens=512, set_size=cfg.set_size, header=header,
                       temperature=cfg.answer_temperature, span_tokens=cfg.read_span_tokens)
    got = region.ask(states, spans, qs, [0, 1, 2])
    assert region.stats["passes"] == 3 and region.stats["asked"] == 12    # one pass per document
    for d in range(3):
        ans, margin = got[(d, 0)]
        assert isinstance(ans, bool) and (margin > 0) == ans
        p, margin = got[(d, 1)]
        assert p == pytest.approx(1 / (1 + math.exp(-margin / cfg.answer_temperature)))
        c, probs = got[(d, 2)]
        assert c in (0, 1, 2) and probs.sum() == pytest.approx(1.0)
        span, _ = got[(d, 3)]
        assert span is None or 0 <= span[0] <= span[1] < len(docs[d])
    # a set size of 2 splits the four questions into two passes per document
    small = SetRegion(m, m.head, chunk_tokens=512, set_size=2, header=header)
    again = small.ask(states, spans, qs, [0])
    assert small.stats["passes"] == 2 and set(again) == {(0, 0), (0, 1), (0, 2), (0, 3)}


def test_sql_on_a_set_attention_model():
    docs = ["the invoice was paid in full on march first", "the parcel arrived broken and late",
            "thanks for the quick reply", "the parcel arrived broken and late"]
    with quail.Session(config=quail.EngineConfig(model="d1-tiny", device="cpu")) as s:
        s.register("t", quail.DocumentProvider.from_table(pa.table({"id": [0, 1, 2, 3], "body": docs}),
                                                          id_col="id"))
        res = s.sql("SELECT id, AI.CLASSIFY(body, ['billing', 'shipping', 'other']) AS kind, "
                    "AI.SCORE(PROMPT('Is {0} urgent?', body)) AS urgency, "
                    "AI.EXTRACT(body, 'What arrived?') AS what, "
                    "AI.IF(PROMPT('Is {0} a complaint?', body)) AS complaint FROM t ORDER BY id").run()
        out = res.table
        assert out.column("kind").to_pylist()[1] == out.column("kind").to_pylist()[3]   # same document
        assert set(out.column("kind").to_pylist()) <= {"billing", "shipping", "other"}
        assert all(0 < u < 1 for u in out.column("urgency").to_pylist())
        assert all(isinstance(c, bool) for c in out.column("complaint").to_pylist())
        region = res.report["regions"][0]
        # three distinct documents, four questions each, all in one pass per document
        assert region["documents"] == 3 and region["asked"] == 12 and region["set_passes"] == 3
        kept = s.sql("SELECT id FROM t WHERE AI.IF(PROMPT('Is {0} a complaint?', body)) AND "
                     "AI.SCORE(PROMPT('Is {0} urgent?', body)) > 0.0").run()
        with pytest.raises(Exception, match="decoding|decodes"):
            s.sql("SELECT AI.MAP(body, 'Summarize') FROM t").collect()
    assert kept.table.num_rows <= 4
