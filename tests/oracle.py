"""A region engine that answers from planted truth, for the SQL-level tests.

`OracleEngine.run_region` has the engine's region semantics (one read per
distinct document and guard inputs; calls asked in order; a dropping filter
that answers FALSE ends the row's chain; a guarded call asked only where its
guard is TRUE) but answers each question from a hash of the question text and
the document instead of a forward pass, and records every question asked.
This is the role of the reference's planted-model oracle
(tests/helpers/oracle.py, planted_model.py): the planner and executor are
the real ones, only the network is replaced.
"""

from __future__ import annotations

import zlib

from quail_b200.api.engine import RegionOutput
from quail_b200.sql import guards as G


def _h(*parts) -> int:
    return zlib.crc32("\x1f".join(str(p) for p in parts).encode())


class OracleEngine:
    cfg = None

    def __init__(self, pass_rate: float = 0.4):
        self.pass_rate = pass_rate
        self.asked: list = []          # (kind, question tail, document)

    # planted truth -------------------------------------------------------
    def answer(self, call, doc):
        h = _h(call.kind, call.tail, doc)
        if call.kind == "filter":
            return (h % 1000) < self.pass_rate * 1000
        if call.kind == "score":
            return (h % 10_000) / 10_000.0
        if call.kind == "classify":
            return call.labels[h % len(call.labels)]
        if call.kind in ("map", "extract"):
            return f"answer-{h % 97}"
        raise ValueError(f"the oracle does not answer {call.kind}")

    def run_region(self, preamble: str, docs: list, calls: list) -> RegionOutput:
        guards = [c.guard for c in calls if c.guard is not None]
        seen: dict = {}
        values = []
        asked = 0
        for i, doc in enumerate(docs):
            key = (doc, tuple(G.signature(g, i) for g in guards))
            if key in seen:
                values.append(dict(seen[key]))
                continue
            got: dict = {}
            for c in calls:
                if c.guard is not None and not G.asks(c.guard, i, got):
                    continue
                v = self.answer(c, doc)
                self.asked.append((c.kind, c.tail, doc))
                asked += 1
                got[c.name] = v
                if c.kind == "filter" and c.drops and not v:
                    break
            seen[key] = got
            values.append(dict(got))
        stats = {"passes": 1 if docs else 0, "fresh_tokens": 0, "documents": len(seen), "rows": len(docs),
                 "asked": asked}
        return RegionOutput(values=values, stats=stats)

    def run_pairs(self, preamble: str, anchors: list, pairs: list, call) -> RegionOutput:
        values = []
        for i, other in pairs:
            v = self.answer(call, anchors[i] + "\x1e" + other)
            self.asked.append((call.kind, call.tail, anchors[i] + "\x1e" + other))
            values.append({call.name: v})
        used = {i for i, _ in pairs}
        stats = {"passes": 1 if pairs else 0, "fresh_tokens": 0, "documents": len(used), "rows": len(pairs),
                 "asked": len(pairs), "anchor_tokens": sum(len(anchors[i]) for i in used)}
        return RegionOutput(values=values, stats=stats)

    def close(self):
        pass
