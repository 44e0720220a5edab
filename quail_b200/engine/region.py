"""Running a chain of AI calls over one table's documents on one GPU.

A region holds the documents (token ids) and an ordered chain of calls; a
call after a filter runs only on the rows that filter kept (the reference's
guards: quail/backends/quail/executor/region.py, model_operator.py and the
operators in operators/filter.py, score.py, classify.py, map.py). For each
row:

  first call   one task: reads the shared instruction prefix, writes the
               document + the call's question, reads out the last token.
  next calls   one task each: reads the prefix and the first task's document
               tokens (borrowed pages), writes only its own question.
               Consecutive non-filter calls run side by side; a filter
               waits for the calls before it.

Readouts:
  filter    max logit over the TRUE spellings > max over FALSE
  score     sigmoid(max TRUE - max FALSE)
  classify  sum over each label's tokens of log p(token | context): the
            question's last row gives log p(first token) against the
            full-vocabulary log-sum-exp; a label of n tokens adds one
            continuation sequence of its first n-1 tokens read out at every
            position (the reference's label trie, label_stages.py)
  map       greedy decoding: each step appends the argmax token to the
            question's own pages until a stop token or max_tokens
            (map_decoder.py); extract decodes after the phrase cue with the
            copy constraint: the best of the readout's top-k tokens that
            continues a verbatim copy of the document (extract/copy.py)
  decision  a decision model's head scores the option rows against the last
            row (filter: Yes > No; score: sigmoid(Yes - No); classify: the
            best label), readout.py:633-728
  letters   a lettered prompt (slot_lm readout): the LM head's logits of the
            option letters at the last row (filter: A (yes) > B (no); score:
            sigmoid(A - B); classify: the option with the largest letter logit),
            readout.py:558-620
  features  SAE features of the residual stream (a model with an SAE returns
            packed [feature ids | strengths] rows): the last token's, or
            with max pooling each feature's largest strength over the row's
            own tokens (sae/encoder.py, sae/max_pooling.py)

The document's pages stay resident until the row's last call has answered
or a filter dropped it.

Document-isolated models (`isolated`): the shared instruction prefix is part
of every document's block (its KV depends on the document, which the block's
tokens read both ways), so there is no shared prefix task; each document is
one bidirectional task, and every call, the first included, is a follow-up
whose own tokens read the block and each other both ways (the reference's
"document_isolated" mask, attention.py:371-375, planning.rs:241-250).
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from functools import partial

import numpy as np

from quail_b200.engine.stage_executor import StageExecutor, Task
from quail_b200.ops.kernels import READOUT_TOPK as TOPK

PREFIX_KEY = ("prefix",)
# QUAIL_EXTRACT_TRACE=<path>: one JSON line per copy-constrained choice (row, step, the readout's
# candidates, the chosen token, how many document positions the copy can continue at)
_EXTRACT_TRACE = os.environ.get("QUAIL_EXTRACT_TRACE")


def _trace_extract(rec: dict) -> None:
    import json
    with open(_EXTRACT_TRACE, "a", encoding="utf-8") as f:
        f.write(json.dumps(rec) + "\n")
DRAFT_TOKENS = 8          # document tokens drafted per pass once a copy has one continuation


@dataclass
class Call:
    """One AI call of the chain, already tokenized."""

    kind: str                      # "filter" | "score" | "classify" | "map" | "extract"
    suffix: np.ndarray             # token ids after the document
    true_cols: list = field(default_factory=list)    # answer-row columns (filter / score)
    false_cols: list = field(default_factory=list)
    labels: list = field(default_factory=list)       # classify: token ids of each label
    label_cols: list = field(default_factory=list)   # classify: answer column of each label token
    max_tokens: int = 256                            # map / extract
    stop_ids: tuple = ()
    name: str = ""
    probabilities: bool = False
    pooling: str = "last"                            # features: "last" token or "max" over the row's tokens
    # decision models: rows read by the decision head, as distances before the
    # last row (one per option, then 0); empty = an LM-head readout
    offsets: tuple = ()
    # extract: every generated token continues a verbatim copy of the row's document
    # (the readout carries the best few tokens; the best one the copy allows wins)
    copy: bool = False
    # filter: a FALSE answer drops the row, so no later call is asked (a WHERE
    # conjunct); False keeps the row and only records the value (a projection)
    drops: bool = True
    # demand guard: when(row, answers so far) decides whether the call is asked on
    # the row at all (None: always); `after` lists the earlier calls it reads
    when: object = None
    after: tuple = ()
    # lettered classify (slot_lm readout): the answer column of each option's letter; the
    # answer is the option whose letter has the largest logit at the last row
    letter_cols: list = field(default_factory=list)
    # map: stop_test(row, tokens so far) -> "continue" | "stop": the answer ends early once a
    # test of it is decided on its text so far (quail_b200.sql.partial)
    stop_test: object = None
    # lettered classify on a canvas model: canvas(row, draw) -> the answer canvas's token ids, a
    # follow-up read both ways after the question; the letters are read at its row 0. A first
    # draw whose label entropy exceeds `entropy` is averaged with draws 1 .. draws-1
    canvas: object = None
    draws: int = 1
    entropy: float = 0.1


@dataclass
class RowResult:
    values: dict = field(default_factory=dict)  # call name -> value
    kept: bool = True


class RegionRun:
    def __init__(self, executor: StageExecutor, prefix: np.ndarray, docs: list, calls: list[Call],
                 doc_ids: list | None = None, answer_width: int | None = None, decision=None,
                 isolated: bool = False):
        self.ex = executor
        self.isolated = isolated              # document-isolated blocks (docs already hold the prefix)
        self.decision = decision              # models.decision.DecisionHead of a decision model
        self.prefix = np.asarray(prefix, dtype=np.int32)
        self.docs = [np.asarray(d, dtype=np.int32) for d in docs]
        self.calls = calls
        self.doc_ids = doc_ids if doc_ids is not None else list(range(len(docs)))
        self.results = [RowResult() for _ in docs]
        self.asked = 0
        self.fresh_tokens = 0
        self.stopped_early = 0                # answers ended once their test was decided
        self._canvas_probs: dict = {}         # (row, call) -> label probabilities of its canvas draws
        self._next = [0] * len(docs)          # next call index to submit per row
        self._pending = [0] * len(docs)       # calls in flight per row
        self._label_parts: dict = {}
        self._copies: dict = {}               # (row, call) -> document positions a copy may continue at
        self.drafted = 0                      # draft tokens accepted (copy-constrained extraction)
        self.progress = None                  # utils.progress.Count advanced as each row finishes
        self.on_finish = None                 # on_finish(r): row r's chain is done (streamed answers)
        # retention across regions: retain_key(r) names row r's document KV for later regions (None:
        # free it); a document found retained is not prefilled again, one whose KV was evicted
        # is recomputed (a replay)
        self.retain_key = None
        self._resident_doc = [False] * len(docs)
        # columns after the answer rows in a full readout: argmax, lse
        self.nans = answer_width

    # ------------------------------------------------------------ geometry
    def _question(self, r: int, ci: int):
        """(own key, reads, position of the first own token, own length) of call ci's question."""
        P = len(self.prefix)
        doc_len = len(self.docs[r])
        if ci == 0 and not self._resident_doc[r]:
            return ("doc", r), [(PREFIX_KEY, P)], P, doc_len + len(self.calls[0].suffix)
        reads = [(PREFIX_KEY, P), (("doc", r), doc_len)] if doc_len else [(PREFIX_KEY, P)]
        if self.isolated:
            reads = [(("doc", r), doc_len)]
        return ("q", r, ci), reads, P + doc_len, len(self.calls[ci].suffix)

    def _full_cols(self, row):
        na = self.nans if self.nans is not None else len(row) - 2
        return na, na + 1

    # ------------------------------------------------------------ readouts
    @staticmethod
    def _margin(call: Call, row) -> float:
        t = max(float(row[c]) for c in call.true_cols)
        f = max(float(row[c]) for c in call.false_cols)
        return t - f

    def _decided(self, r: int, ci: int, rows) -> None:
        """A decision head's answer: option scores (No, Yes for a filter or score; the labels for classify)."""
        call = self.calls[ci]
        res = self.results[r]
        scores = self.decision.combine(rows)
        if call.kind == "filter":
            keep = bool(scores[1] > scores[0])
            res.values[call.name] = keep
            if not keep and call.drops:
                res.kept = False
        elif call.kind == "score":
            res.values[call.name] = 1.0 / (1.0 + math.exp(-(float(scores[1]) - float(scores[0]))))
        else:
            res.values[call.name] = int(np.argmax(scores))
            if call.probabilities:
                e = np.exp(scores - scores.max())
                res.values[call.name + "#probs"] = [float(x) for x in e / e.sum()]
        self.asked += 1
        self._finish_call(r, ci)

    def _answered(self, r: int, ci: int, row) -> None:
        call = self.calls[ci]
        res = self.results[r]
        if call.offsets:
            self._decided(r, ci, row)
            return
        if call.kind == "filter":
            keep = self._margin(call, row) > 0
            res.values[call.name] = bool(keep)
            if not keep and call.drops:
                res.kept = False
            self._finish_call(r, ci)
        elif call.kind == "score":
            res.values[call.name] = 1.0 / (1.0 + math.exp(-self._margin(call, row)))
            self._finish_call(r, ci)
        elif call.kind == "classify" and call.letter_cols:
            scores = np.asarray([float(row[c]) for c in call.letter_cols], dtype=np.float64)
            res.values[call.name] = int(np.argmax(scores))
            if call.probabilities:
                e = np.exp(scores - scores.max())
                res.values[call.name + "#probs"] = [float(x) for x in e / e.sum()]
            self._finish_call(r, ci)
        elif call.kind == "classify":
            self._classify_first(r, ci, row)
        elif call.kind in ("map", "extract"):
            self._decode_step(r, ci, row, [])
        elif call.kind == "features":
            res.values[call.name] = feature_list(row)
            self._finish_call(r, ci)
        self.asked += 1

    def _classify_first(self, r, ci, row):
        call = self.calls[ci]
        _, lse_col = self._full_cols(row)
        lse = float(row[lse_col])
        scores = [float(row[cols[0]]) - lse for cols in call.label_cols]
        waiting = [li for li, lab in enumerate(call.labels) if len(lab) > 1]
        self._label_parts[(r, ci)] = [scores, len(waiting)]
        if not waiting:
            self._classify_done(r, ci)
            return
        key, reads, pos, own_len = self._question(r, ci)
        for li in waiting:
            lab = np.asarray(call.labels[li], dtype=np.int32)
            toks = lab[:-1]
            self.fresh_tokens += len(toks)
            self.ex.submit(Task(np_rows=True, key=("lab", r, ci, li), tokens=toks, pos_start=pos + own_len,
                                reads=reads + [(key, own_len)], readout=True,
                                readout_rows=tuple(range(len(toks))), full_readout=True,
                                on_done=lambda t, rows, r=r, ci=ci, li=li: self._label_rows(r, ci, li, rows)))

    def _label_rows(self, r, ci, li, rows):
        call = self.calls[ci]
        parts = self._label_parts[(r, ci)]
        _, lse_col = self._full_cols(rows[0])
        for j in range(rows.shape[0]):
            col = call.label_cols[li][j + 1]
            parts[0][li] += float(rows[j][col]) - float(rows[j][lse_col])
        parts[1] -= 1
        if parts[1] == 0:
            self._classify_done(r, ci)

    def _classify_done(self, r, ci):
        call = self.calls[ci]
        scores, _ = self._label_parts.pop((r, ci))
        best = int(np.argmax(scores))
        res = self.results[r]
        res.values[call.name] = best
        if call.probabilities:
            m = max(scores)
            e = [math.exp(s - m) for s in scores]
            z = sum(e)
            res.values[call.name + "#probs"] = [x / z for x in e]
        self._finish_call(r, ci)

    def _decode_step(self, r, ci, row, generated, draft=()):
        """One decode step of row r's call ci; `generated` is the row's token list (appended in place).

        `row` holds one readout row, or with a draft one per drafted position: the
        draft's tokens are kept while the step's choice (greedy, or the copy
        constraint's) agrees with them, and the first disagreeing choice (or the
        choice after the whole draft) is the step's new token.
        """
        call = self.calls[ci]
        vals = np.asarray(row.numpy() if hasattr(row, "numpy") else row)
        rows = vals.reshape(-1, vals.shape[-1])
        arg_col = self.nans if self.nans is not None else (rows.shape[1] - 2 - (2 * TOPK if call.copy else 0))
        tok = -1
        for jrow in range(rows.shape[0]):
            tok = (self._copy_choice(r, ci, rows[jrow], arg_col, generated) if call.copy
                   else int(round(float(rows[jrow][arg_col]))))
            if (jrow < len(draft) and tok == draft[jrow] and tok not in call.stop_ids
                    and len(generated) + 1 < call.max_tokens):
                generated.append(tok)
                self.drafted += 1
                continue
            break
        stop = tok < 0 or tok in call.stop_ids
        if not stop:
            generated.append(tok)
            if (call.stop_test is not None and len(generated) < call.max_tokens
                    and call.stop_test(r, generated) == "stop"):
                stop = True
                self.stopped_early += 1
        if stop or len(generated) >= call.max_tokens:
            self.results[r].values[call.name] = generated
            self._copies.pop((r, ci), None)
            self._finish_call(r, ci)
            return
        key, reads, pos, own_len = self._question(r, ci)
        n_prev = len(generated) - 1
        nxt = self._draft(r, ci, call.max_tokens - len(generated)) if call.copy else ()
        self.fresh_tokens += 1 + len(nxt)
        self.ex.submit_continuation(Task(np_rows=True, key=key, tokens=[tok, *nxt], pos_start=pos + own_len + n_prev, reads=reads,
                                         readout=True, full_readout=True, own_prefix=own_len + n_prev,
                                         free_after=False, topk=call.copy,
                                         readout_rows=tuple(range(1 + len(nxt))) if nxt else None,
                                         on_done=partial(self._decode_next, r, ci, generated, nxt)))

    def _decode_next(self, r, ci, generated, draft, task, row):
        self._decode_step(r, ci, row, generated, draft)

    def _draft(self, r, ci, room: int) -> tuple:
        """Document-copy draft: when the copy so far continues at one document position only,
        the next few document tokens, to verify in one pass (reference: extract/candidates.py)."""
        state = self._copies.get((r, ci))
        doc = self.docs[r]
        if state is None or state.size != 1 or state[0] >= len(doc):
            return ()
        p = int(state[0])
        n = min(DRAFT_TOKENS, room, len(doc) - p)
        return tuple(int(t) for t in doc[p:p + n]) if n > 0 else ()

    def _copy_choice(self, r, ci, vals, arg_col, generated) -> int:
        """The next token of a copy-constrained extraction: the best-ranked readout candidate
        that continues a verbatim copy of the document (any document token to start), or a
        stop token; when no candidate qualifies, the phrase ends.

        The copy state is the set of document positions that can follow the phrase so far
        (the reference's copy-constrained extraction: executor/extract/copy.py).
        """
        call = self.calls[ci]
        doc = self.docs[r]
        state = self._copies.get((r, ci))
        if state is None:
            state = np.arange(len(doc))               # nothing copied yet: any position starts
        cand = vals[arg_col + 2:arg_col + 2 + TOPK].astype(np.int64)
        allowed = doc[state[state < len(doc)]]
        choice, kept = (call.stop_ids[0] if call.stop_ids else -1), 0
        for t in cand:
            t = int(t)
            if t in call.stop_ids:
                choice = t
                break
            hit = state[(state < len(doc)) & (allowed == t)]
            if hit.size:
                self._copies[(r, ci)] = hit + 1
                choice, kept = t, int(hit.size)
                break
        if _EXTRACT_TRACE:
            _trace_extract({"row": int(r), "call": self.calls[ci].name, "step": len(generated),
                            "candidates": [int(t) for t in cand], "chosen": int(choice), "positions": kept})
        return choice

    # ------------------------------------------------------------ scheduling
    def _finish_call(self, r: int, ci: int) -> None:
        if ci > 0 or self._resident_doc[r]:
            self.ex.free(("q", r, ci))
        elif self.calls[0].kind in ("map", "extract") and len(self.calls) > 1 and not self.ex.pool.state_slots:
            # KV rewind: the first call decoded into the document's own pages; the later
            # questions read only the document, so its generated tokens' pages go back
            self.ex.rewind(("doc", r), len(self.docs[r]))
        for li in range(len(self.calls[ci].labels)):
            if self.ex.pool.resident(("lab", r, ci, li)):
                self.ex.free(("lab", r, ci, li))
        self._pending[r] -= 1
        if self._pending[r] == 0:
            self._advance(r)

    @staticmethod
    def _barrier(call: Call) -> bool:
        return call.kind == "filter" and call.drops

    def _asks(self, r: int, ci: int) -> bool:
        when = self.calls[ci].when
        return when is None or bool(when(r, self.results[r].values))

    def _advance(self, r: int) -> None:
        res = self.results[r]
        while True:
            ci = self._next[r]
            if not res.kept or ci >= len(self.calls):
                if self.ex.pool.resident(("doc", r)):
                    keep = self.retain_key(r) if self.retain_key is not None else None
                    if keep is not None and not self.ex.pool.state_slots and len(self.docs[r]):
                        self.ex.rewind(("doc", r), len(self.docs[r]))
                        self.ex.retain(("doc", r), keep)
                    else:
                        self.ex.free(("doc", r))
                if self.progress is not None:
                    self.progress.advance()
                if self.on_finish is not None:
                    self.on_finish(r)
                return
            # a dropping filter runs alone; other calls up to the next one run side by
            # side, except a call whose guard reads an answer of the same batch
            batch = [ci]
            if not self._barrier(self.calls[ci]):
                j = ci + 1
                while (j < len(self.calls) and not self._barrier(self.calls[j])
                       and not set(self.calls[j].after) & set(batch)):
                    batch.append(j)
                    j += 1
            self._next[r] = batch[-1] + 1
            ask = [c for c in batch if self._asks(r, c)]
            if not ask:
                continue
            self._pending[r] = len(ask)
            for c in ask:
                self._submit_question(r, c)
            return

    @staticmethod
    def _pooled_rows(call: Call, n: int):
        """Readout offsets: every own token for max-pooled features, the option rows and the
        last row for a decision head, else the last token only."""
        if call.offsets:
            return tuple(n - 1 - o for o in call.offsets)
        return tuple(range(n)) if call.kind == "features" and call.pooling == "max" else None

    @staticmethod
    def _reserve(call: Call) -> int:
        """Decode headroom: a decoding call's generated tokens land in its own pages."""
        return call.max_tokens if call.kind in ("map", "extract") else 0

    def _needs_full(self, call: Call) -> bool:
        return call.kind in ("classify", "map", "extract") and not call.offsets and not call.letter_cols

    def _submit_question(self, r: int, ci: int) -> None:
        call = self.calls[ci]
        key, reads, pos, own_len = self._question(r, ci)
        self.fresh_tokens += len(call.suffix)
        if call.canvas is not None:
            # the question is prefilled without a readout; the answer canvas reads it
            self.ex.submit(Task(np_rows=True, key=key, tokens=call.suffix, pos_start=pos, reads=reads, readout=False,
                                on_done=lambda t, row, r=r, ci=ci: self._canvas_draws(r, ci, (0,)),
                                free_after=False))
            return
        self.ex.submit(Task(np_rows=True, key=key, tokens=call.suffix, pos_start=pos, reads=reads, readout=True,
                            full_readout=self._needs_full(call), reserve_tokens=self._reserve(call), topk=call.copy,
                            readout_rows=self._pooled_rows(call, len(call.suffix)), bidirectional=self.isolated,
                            on_done=lambda t, row, r=r, ci=ci: self._answered(r, ci, row), free_after=False))

    def _canvas_draws(self, r: int, ci: int, draws) -> None:
        """Submit answer canvases `draws` of row r's call ci: each a follow-up of the question
        (prompt, document, question), its rows read both ways, read out at its row 0."""
        call = self.calls[ci]
        key, reads, pos, own_len = self._question(r, ci)
        for d in draws:
            toks = call.canvas(r, d)
            self.fresh_tokens += len(toks)
            self.ex.submit(Task(np_rows=True, key=("cv", r, ci, d), tokens=toks, pos_start=pos + own_len,
                                             reads=reads + [(key, own_len)], readout=True, readout_rows=(0,),
                                             bidirectional=True, free_after=True,
                                             on_done=lambda t, row, r=r, ci=ci, d=d: self._canvas_read(r, ci, d, row)))

    def _canvas_read(self, r: int, ci: int, draw: int, row) -> None:
        call = self.calls[ci]
        res = self.results[r]
        vals = np.asarray(row, dtype=np.float64).reshape(-1)
        scores = np.asarray([vals[c] for c in call.letter_cols])
        e = np.exp(scores - scores.max())
        p = e / e.sum()
        acc = self._canvas_probs.setdefault((r, ci), [])
        acc.append(p)
        if draw == 0:
            entropy = float(-(p * np.log(np.maximum(p, 1e-30))).sum())
            if call.draws > 1 and entropy > call.entropy:
                self._canvas_draws(r, ci, range(1, call.draws))
                return
        elif len(acc) < call.draws:
            return
        mean = np.mean(self._canvas_probs.pop((r, ci)), axis=0)
        res.values[call.name] = int(np.argmax(mean))
        if call.probabilities:
            res.values[call.name + "#probs"] = [float(x) for x in mean]
        self.asked += 1
        self._finish_call(r, ci)

    def _submit_isolated(self) -> None:
        """Every document as one block read both ways; then its calls, all as follow-ups."""
        for r, doc in enumerate(self.docs):
            self._resident_doc[r] = True
            self._next[r] = 0
            if self.retain_key is not None and not self.ex.pool.state_slots:
                rk = self.retain_key(r)
                if rk is not None and self.ex.pool.resident(rk) and self.ex.claim(rk, ("doc", r)):
                    self.ex.stats.reused += 1
                    self._advance(r)
                    continue
                if rk is not None and rk in self.retained_earlier:
                    self.ex.stats.replays += 1
            self._pending[r] = 1
            self.fresh_tokens += len(doc)
            self.ex.submit(Task(np_rows=True, key=("doc", r), tokens=doc, pos_start=0, reads=[], free_after=False,
                                bidirectional=True, on_done=lambda t, row, r=r: self._doc_only(r)))

    def submit_all(self) -> None:
        if self.isolated:
            self._submit_isolated()
            return
        P = len(self.prefix)
        self.fresh_tokens += P
        self.ex.submit(Task(np_rows=True, key=PREFIX_KEY, tokens=self.prefix, pos_start=0, free_after=False))
        first = self.calls[0]
        pinned, cap = 0, self.ex.pool.num_pages // 2
        # a first call that reads every own token (max-pooled features) needs the document computed
        reusable = not (first.kind == "features" and first.pooling == "max")
        for r, doc in enumerate(self.docs):
            if self.retain_key is not None and reusable and len(doc) and not self.ex.pool.state_slots:
                rk = self.retain_key(r)
                if rk is not None and self.ex.pool.resident(rk):
                    need = self.ex.pool.pages_needed(len(doc))
                    if pinned + need <= cap and self.ex.claim(rk, ("doc", r)):
                        # this document's KV is already in the arena: only its questions run
                        pinned += need
                        self._resident_doc[r] = True
                        self.ex.stats.reused += 1
                        self._next[r] = 0
                        self._pending[r] = 0
                        self._advance(r)
                        continue
                elif rk is not None and rk in self.retained_earlier:
                    # retained by an earlier region, evicted since: computed again
                    self.ex.stats.replays += 1
            if not self._asks(r, 0):
                # the first call is not asked on this row: its document alone, then the rest
                self._next[r] = 1
                self._pending[r] = 1
                if len(doc) == 0:
                    self._pending[r] = 0
                    self._advance(r)
                    continue
                self.fresh_tokens += len(doc)
                self.ex.submit(Task(np_rows=True, key=("doc", r), tokens=doc, pos_start=P,
                                    reads=[(PREFIX_KEY, P)], free_after=False,
                                    on_done=lambda t, row, r=r: self._doc_only(r)))
                continue
            toks = np.concatenate([doc, first.suffix])
            self.fresh_tokens += len(toks)
            self._next[r] = 1
            self._pending[r] = 1
            self.ex.submit(Task(np_rows=True, key=("doc", r), tokens=toks, pos_start=P, reads=[(PREFIX_KEY, P)], readout=True,
                                full_readout=self._needs_full(first), reserve_tokens=self._reserve(first),
                                topk=first.copy,
                                readout_rows=self._pooled_rows(first, len(toks)),
                                on_done=lambda t, row, r=r: self._answered(r, 0, row), free_after=False))

    def _doc_only(self, r: int) -> None:
        self._pending[r] = 0
        self._advance(r)

    retained_earlier: frozenset = frozenset()   # keys earlier regions retained (to count replays)

    def run(self):
        self.submit_all()
        self.ex.run()
        if self.ex.pool.resident(PREFIX_KEY):
            self.ex.free(PREFIX_KEY)
        return self.results


def feature_list(rows) -> list:
    """Packed SAE readout rows ([k ids | k strengths] each) -> [(feature, strength)], strongest first.

    One row: its nonzero features. Several rows (max pooling over tokens):
    each feature's largest strength over the rows.
    """
    a = np.asarray(rows, dtype=np.float32)
    a = a.reshape(-1, a.shape[-1])
    k = a.shape[1] // 2
    ids = a[:, :k].astype(np.int64).ravel()
    st = a[:, k:].ravel()
    keep = st > 0
    ids, st = ids[keep], st[keep]
    if ids.size == 0:
        return []
    order = np.lexsort((-st, ids))            # by feature, strongest first within a feature
    ids, st = ids[order], st[order]
    first = np.ones(ids.size, dtype=bool)
    first[1:] = ids[1:] != ids[:-1]
    ids, st = ids[first], st[first]
    by = np.lexsort((ids, -st))              # strongest first, lower id on ties
    return [(int(i), float(v)) for i, v in zip(ids[by], st[by])]


class PairRun:
    """An AI join's questions: every (anchor document, other document) pair, asked once.

    Each anchor document is prefilled once, after the shared prefix; each pair
    is one follow-up task that reads the prefix and its anchor's pages and
    computes only its own tokens (the other document, then the call's
    question), with its answer read at the last token. An anchor's pages are
    freed when its last pair is answered. This is the reference's join
    operator with pair lists (quail/backends/quail/executor/operators/
    join.py:47-739): the anchor side's KV is shared by all of its pairs.
    """

    def __init__(self, executor: StageExecutor, prefix: np.ndarray, anchors: list, pairs: list, call: Call,
                 answer_width: int | None = None):
        self.ex = executor
        self.prefix = np.asarray(prefix, dtype=np.int32)
        self.anchors = [np.asarray(a, dtype=np.int32) for a in anchors]
        self.pairs = [(int(i), np.asarray(t, dtype=np.int32)) for i, t in pairs]
        self.call = call
        self.values: list = [None] * len(self.pairs)
        self.asked = 0
        self.fresh_tokens = 0
        self._left = [0] * len(self.anchors)
        for i, _ in self.pairs:
            self._left[i] += 1
        self.progress = None

    def _answered(self, j: int, row) -> None:
        call = self.call
        margin = RegionRun._margin(call, row)
        self.values[j] = bool(margin > 0) if call.kind == "filter" else 1.0 / (1.0 + math.exp(-margin))
        self.asked += 1
        self.ex.free(("pair", j))
        i = self.pairs[j][0]
        self._left[i] -= 1
        if self._left[i] == 0 and self.ex.pool.resident(("anc", i)):
            self.ex.free(("anc", i))
        if self.progress is not None:
            self.progress.advance()

    def run(self) -> list:
        if self.call.kind not in ("filter", "score"):
            raise ValueError(f"an AI join asks filter or score questions, not {self.call.kind}")
        P = len(self.prefix)
        self.fresh_tokens += P
        self.ex.submit(Task(np_rows=True, key=PREFIX_KEY, tokens=self.prefix, pos_start=0, free_after=False))
        for i, a in enumerate(self.anchors):
            if self._left[i] and len(a):
                self.fresh_tokens += len(a)
                self.ex.submit(Task(np_rows=True, key=("anc", i), tokens=a, pos_start=P, reads=[(PREFIX_KEY, P)],
                                    free_after=False))
        for j, (i, toks) in enumerate(self.pairs):
            a_len = len(self.anchors[i])
            own = np.concatenate([toks, self.call.suffix]).astype(np.int32)
            reads = [(PREFIX_KEY, P)] + ([(("anc", i), a_len)] if a_len else [])
            self.fresh_tokens += len(own)
            self.ex.submit(Task(np_rows=True, key=("pair", j), tokens=own, pos_start=P + a_len, reads=reads,
                                readout=True, free_after=False,
                                on_done=lambda t, row, j=j: self._answered(j, row)))
        self.ex.run()
        self.ex.free(PREFIX_KEY)
        return self.values
