"""Running a chain of AI calls over one table's documents on one GPU.

A region holds the documents (token ids) and an ordered chain of calls; a
call after a filter runs only on the rows that filter kept (the reference's
guards: quail/backends/quail/executor/region.py, model_operator.py,
operators/filter.py, score.py). For every row:

  first call   one task: reads the shared instruction prefix, writes
               document + question, reads out the last token.
  next calls   one task each: reads the prefix and the first call's
               document tokens (borrowed pages), writes only the question.

The document's pages stay resident until the row's last call has answered
or a filter dropped it. Readouts: a filter compares the max logit over the
TRUE spellings with the max over FALSE; a score is sigmoid(true - false).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from quail_b200.engine.stage_executor import StageExecutor, Task

PREFIX_KEY = ("prefix",)


@dataclass
class Call:
    """One AI call of the chain, already tokenized."""

    kind: str                      # "filter" | "score" | "classify"
    suffix: np.ndarray             # token ids after the document
    true_cols: list = field(default_factory=list)    # answer-row columns (filter/score)
    false_cols: list = field(default_factory=list)
    label_cols: list = field(default_factory=list)   # classify: column of each label's first token
    name: str = ""


@dataclass
class RowResult:
    values: dict = field(default_factory=dict)  # call name -> value
    kept: bool = True


class RegionRun:
    def __init__(self, executor: StageExecutor, prefix: np.ndarray, docs: list[np.ndarray], calls: list[Call],
                 doc_ids: list | None = None):
        self.ex = executor
        self.prefix = np.asarray(prefix, dtype=np.int32)
        self.docs = docs
        self.calls = calls
        self.doc_ids = doc_ids if doc_ids is not None else list(range(len(docs)))
        self.results = [RowResult() for _ in docs]
        self.asked = 0
        self.fresh_tokens = 0

    # ------------------------------------------------------------ readouts
    @staticmethod
    def _filter_margin(call: Call, row) -> float:
        t = max(float(row[c]) for c in call.true_cols)
        f = max(float(row[c]) for c in call.false_cols)
        return t - f

    def _answer(self, r: int, ci: int, row) -> None:
        call = self.calls[ci]
        res = self.results[r]
        if call.kind == "filter":
            keep = self._filter_margin(call, row) > 0
            res.values[call.name] = bool(keep)
            if not keep:
                res.kept = False
        elif call.kind == "score":
            m = self._filter_margin(call, row)
            res.values[call.name] = 1.0 / (1.0 + math.exp(-m))
        elif call.kind == "classify":
            scores = [float(row[c]) for c in call.label_cols]
            res.values[call.name] = int(np.argmax(scores))
        self.asked += 1
        nxt = ci + 1
        if res.kept and nxt < len(self.calls):
            self._submit_followup(r, nxt)
        else:
            self.ex.free(("doc", r))

    # ------------------------------------------------------------ tasks
    def _submit_followup(self, r: int, ci: int) -> None:
        doc_len = len(self.docs[r])
        call = self.calls[ci]
        P = len(self.prefix)
        self.fresh_tokens += len(call.suffix)
        self.ex.submit(Task(key=("q", r, ci), tokens=call.suffix, pos_start=P + doc_len,
                            reads=[(PREFIX_KEY, P), (("doc", r), doc_len)], readout=True,
                            on_done=lambda t, row, r=r, ci=ci: self._answer(r, ci, row), free_after=True))

    def submit_all(self) -> None:
        P = len(self.prefix)
        self.fresh_tokens += P
        self.ex.submit(Task(key=PREFIX_KEY, tokens=self.prefix, pos_start=0, free_after=False))
        first = self.calls[0]
        for r, doc in enumerate(self.docs):
            toks = np.concatenate([np.asarray(doc, dtype=np.int32), first.suffix])
            self.fresh_tokens += len(toks)
            self.ex.submit(Task(key=("doc", r), tokens=toks, pos_start=P, reads=[(PREFIX_KEY, P)], readout=True,
                                on_done=lambda t, row, r=r: self._answer(r, 0, row), free_after=False))

    def run(self):
        self.submit_all()
        self.ex.run()
        self.ex.free(PREFIX_KEY)
        return self.results
