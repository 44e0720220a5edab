"""Set-attention regions: every question about a document asked in passes over that document.

Under set attention (LFM3 / d1) nothing is kept between passes: a pass is the
document's state (prompt head, document, state tail) followed by up to the
model's set size of questions, and the state reads its questions (the
reference's set passes: quail/backends/quail/executor/set_passes.py,
pass_groups.py, operators/set_classify.py, set_extract.py). The calls of a
region are split into pass groups: a filter that drops rows ends a group (the
next group asks only the rows it kept) and so does a call whose demand guard
reads an answer of the same group. In a group every document gets one pass,
or more when its questions exceed the set size or a chunk.

Answers (readout rows are final-normed hidden states; `targets` the output
head's rows of the answer tokens):
  yes / no   the question's last row: max over the yes spellings' logits minus
             max over the no spellings' (filter: > 0; score: sigmoid(margin / T))
  choice     the last row: each option's best spelling logit / T, softmaxed;
             the answer is the likeliest option
  read       two slot rows ("start:", "end:") point at the document rows (row 0,
             the token before the document, stands for nothing): scores are dot
             products over sqrt(width), log-softmaxed; P(found) = 1 - P(start
             at row 0), calibrated through the model's knots; the span is the
             best start + end at most `read_span_tokens` rows apart
             (readout.py:376-426, operators/set_extract.py)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from quail_b200.models.lfm3 import SetPass

# the d1 layout's question header (crates/quail-planner/src/prompts.rs:174-189): it ends the
# state (the state tail) and opens every question after a pass's first
D1_HEADER = "\n\n\nQUESTION:\n"


@dataclass
class SetQuestion:
    """One call's question in set passes, tokenized."""

    kind: str                       # "yes_no" | "score" | "choice" | "read"
    body: np.ndarray                # the question's tokens after its header
    name: str = ""
    yes: list = field(default_factory=list)      # answer-token ids (yes_no / score)
    no: list = field(default_factory=list)
    options: list = field(default_factory=list)  # choice: per option, its spellings' token ids
    slots: tuple = (0,)             # rows read, counted back from the question's last row
    drops: bool = True
    when: object = None             # demand guard: when(row, answers so far)
    after: tuple = ()


def split_passes(state: int, lengths: list, header: int, set_size: int, budget: int) -> list[list]:
    """Question indices per pass, in order: at most set_size questions, the state and the
    questions (each after the first with its header) within the token budget.

    Raises:
        ValueError: one question does not fit a pass with the state.
    """
    passes, cur, used = [], [], state
    for i, n in enumerate(lengths):
        if state + n > budget:
            raise ValueError(f"a {n}-token question does not fit one {budget}-token pass with its "
                             f"{state}-token state")
        extra = n + (header if cur else 0)
        if cur and (len(cur) == set_size or used + extra > budget):
            passes.append(cur)
            cur, used = [], state
            extra = n
        cur.append(i)
        used += extra
    if cur:
        passes.append(cur)
    return passes


def calibrated(knots, value: float) -> float:
    """A raw value through increasing (raw, calibrated) knots: linear between, flat past the ends."""
    if not knots:
        return float(value)
    raw, out = zip(*knots)
    return float(np.interp(value, raw, out))


def pointer_span(start_row: torch.Tensor, end_row: torch.Tensor, doc_rows: torch.Tensor, span_tokens: int):
    """(first row, last row, raw P(found)) of one read: rows counted from the document's
    first token plus one, (0, 0) for nothing."""
    W = doc_rows.shape[0]
    scale = 1.0 / math.sqrt(doc_rows.shape[1])
    s = torch.log_softmax((doc_rows @ start_row) * scale, dim=0)
    e = torch.log_softmax((doc_rows @ end_row) * scale, dim=0)
    found = float(-torch.expm1(s[0]))
    if W == 1 or found < 0.5:
        return 0, 0, found
    cap = max(1, min(span_tokens or W, W - 1))
    # best start i >= 1 and end j in [i, i + cap - 1]
    n = W - 1
    ss, ee = s[1:], e[1:]
    best, bi, bj = -math.inf, 0, 0
    # a banded search: for each offset d in [0, cap) the pair (i, i + d)
    for d in range(min(cap, n)):
        tot = ss[:n - d] + ee[d:]
        k = int(torch.argmax(tot))
        v = float(tot[k])
        if v > best:
            best, bi, bj = v, k, k + d
    return bi + 1, bj + 1, found


class SetRegion:
    """Runs one region's questions over its documents in set-attention passes."""

    def __init__(self, model, head: torch.Tensor, chunk_tokens: int, set_size: int, header: np.ndarray,
                 temperature: float = 1.0, span_tokens: int = 0, found_knots=()):
        self.model = model
        self.head = head                  # [V, H] output head (bf16 or fp32)
        self.chunk_tokens = chunk_tokens
        self.set_size = max(1, set_size)
        self.header = np.asarray(header, dtype=np.int32)
        self.temperature = temperature
        self.span_tokens = span_tokens
        self.found_knots = tuple(found_knots)
        self.stats = {"passes": 0, "chunks": 0, "fresh_tokens": 0, "asked": 0}

    # ------------------------------------------------------------ passes
    def _passes_for(self, state: np.ndarray, doc_start: int, doc_len: int, qs: list[SetQuestion]):
        """The passes asking `qs` of one document, and per question (pass index, read rows)."""
        lengths = [len(q.body) for q in qs]
        groups = split_passes(len(state), lengths, len(self.header), self.set_size, self.chunk_tokens)
        out, where = [], {}
        for g in groups:
            toks = [state]
            rows, qlens = [], []
            row = len(state)
            for k, qi in enumerate(g):
                body = qs[qi].body if k == 0 else np.concatenate([self.header, qs[qi].body])
                toks.append(body)
                last = row + len(body) - 1
                q_rows = [last - off for off in qs[qi].slots]
                where[qi] = (len(out), len(rows), len(q_rows))
                rows.extend(q_rows)
                qlens.append(len(body))
                row += len(body)
            if any(qs[qi].kind == "read" for qi in g):
                # the document rows a read points at: the token before the document, then the document
                first = len(rows)
                rows.extend(range(doc_start - 1, doc_start + doc_len))
                for qi in g:
                    where[qi] = where[qi] + (first,)
            out.append(SetPass(tokens=np.concatenate(toks).astype(np.int32), state=len(state), questions=qlens,
                               read_rows=rows))
        return out, where

    def _run(self, passes: list[SetPass]) -> list[torch.Tensor]:
        """Every pass's read rows, in chunks of at most chunk_tokens tokens."""
        out: list = []
        i = 0
        while i < len(passes):
            j, used = i, 0
            while j < len(passes) and (j == i or used + passes[j].length <= self.chunk_tokens):
                used += passes[j].length
                j += 1
            out.extend(self.model.forward_passes(passes[i:j]))
            self.stats["chunks"] += 1
            self.stats["fresh_tokens"] += used
            i = j
        self.stats["passes"] += len(passes)
        return out

    # ------------------------------------------------------------ answers
    def _answer(self, q: SetQuestion, rows: torch.Tensor, doc_rows: torch.Tensor | None):
        head = self.head
        if q.kind in ("yes_no", "score"):
            ids = torch.as_tensor(q.yes + q.no, dtype=torch.long, device=head.device)
            logits = (rows[-1:].to(head.dtype) @ head.index_select(0, ids).t()).float()[0]
            margin = float(logits[:len(q.yes)].max() - logits[len(q.yes):].max())
            if q.kind == "yes_no":
                return margin > 0, margin
            return 1.0 / (1.0 + math.exp(-margin / self.temperature)), margin
        if q.kind == "choice":
            flat = [t for sp in q.options for t in sp]
            ids = torch.as_tensor(flat, dtype=torch.long, device=head.device)
            logits = (rows[-1:].to(head.dtype) @ head.index_select(0, ids).t()).float()[0].cpu().numpy()
            scores, k = [], 0
            for sp in q.options:
                scores.append(float(logits[k:k + len(sp)].max()))
                k += len(sp)
            z = np.asarray(scores) / self.temperature
            p = np.exp(z - z.max())
            p /= p.sum()
            return int(np.argmax(p)), p
        # read: start slot then end slot
        first, last, found = pointer_span(rows[0].float(), rows[1].float(), doc_rows.float(), self.span_tokens)
        cal = calibrated(self.found_knots, found)
        if first == 0 or cal < 0.5:
            return None, cal
        return (first - 1, last - 1), cal

    def ask(self, states: list, doc_spans: list, qs: list[SetQuestion], who: list) -> dict:
        """Ask `qs` of the documents `who` (indices into states); returns {(doc, question): answer}."""
        passes, index = [], []
        for d in who:
            ps, where = self._passes_for(states[d], doc_spans[d][0], doc_spans[d][1], qs)
            index.append((d, len(passes), where))
            passes.extend(ps)
        rows = self._run(passes)
        out = {}
        for d, base, where in index:
            for qi, w in where.items():
                r = rows[base + w[0]]
                slot = r[w[1]:w[1] + w[2]]
                doc_rows = r[w[3]:] if len(w) > 3 else None
                out[(d, qi)] = self._answer(qs[qi], slot, doc_rows)
                self.stats["asked"] += 1
        return out
