"""AI calls of one query written almost the same.

A query asks the model once for calls written the same way (they share a node
key). Two calls that differ only slightly are most likely one call written
twice by mistake, and the model would answer both, maybe differently:

  spelling  the same function over the same columns and options, whose texts
            differ only in case, whitespace or punctuation: refused, with both
            texts in the message;
  typo      texts of at least 12 characters at most two letter edits apart with
            the same digits: kept, with a warning in the query report.

Texts that differ in a digit ('from 2027' / 'from 2028') are different calls.
Reference: crates/quail-datafusion/src/derive/similar.rs (the same two
likenesses and thresholds; the comparison here is this build's own).
"""

from __future__ import annotations

import json
import re

TYPO_MIN_CHARS = 12
TYPO_MAX_EDITS = 2


def _texts(node) -> list[str]:
    """The string literals of a call, in order (prompt templates, labels, questions)."""
    out = []

    def visit(n):
        if isinstance(n, dict):
            if n.get("type") == "literal" and n.get("kind") == "string":
                out.append(n["value"])
            for v in n.values():
                visit(v)
        elif isinstance(n, list):
            for v in n:
                visit(v)
    visit(node)
    return out


def _shape(node) -> str:
    """The call with every string literal blanked: two calls of one shape read the same columns
    with the same options and differ, if at all, in their texts."""
    def blank(n):
        if isinstance(n, dict):
            if n.get("type") == "literal" and n.get("kind") == "string":
                return {"type": "literal", "kind": "string", "value": ""}
            return {k: blank(v) for k, v in n.items()}
        if isinstance(n, list):
            return [blank(v) for v in n]
        return n
    return json.dumps(blank(node), sort_keys=True)


def _spelling(text: str) -> str:
    return re.sub(r"[\W_]+", "", text.lower())


def _edits(a: str, b: str, cap: int) -> int:
    """Levenshtein distance of a and b, stopping once it exceeds cap."""
    if abs(len(a) - len(b)) > cap:
        return cap + 1
    prev = list(range(len(b) + 1))
    for i, ca in enumerate(a, 1):
        cur = [i] + [0] * len(b)
        best = cur[0]
        for j, cb in enumerate(b, 1):
            cur[j] = min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (ca != cb))
            best = min(best, cur[j])
        if best > cap:
            return cap + 1
        prev = cur
    return prev[-1]


def likeness(a: str, b: str) -> str | None:
    """"spelling", "typo" or None for two texts of calls of one shape."""
    if a == b:
        return None
    if _spelling(a) == _spelling(b):
        return "spelling"
    if (min(len(a), len(b)) >= TYPO_MIN_CHARS and re.findall(r"\d", a) == re.findall(r"\d", b)
            and _edits(a.lower(), b.lower(), TYPO_MAX_EDITS) <= TYPO_MAX_EDITS):
        return "typo"
    return None


def similar_calls(calls: list[dict]) -> list[tuple[str, str, str]]:
    """(likeness, first text, second text) of every pair of distinct calls written almost the same."""
    seen: dict = {}
    out = []
    for c in calls:
        key = json.dumps(c, sort_keys=True)
        shape = _shape(c)
        for other_key, other in seen.get(shape, {}).items():
            if other_key == key:
                continue
            for ta, tb in zip(_texts(other), _texts(c)):
                kind = likeness(ta, tb)
                if kind is not None:
                    out.append((kind, ta, tb))
                    break
        seen.setdefault(shape, {})[key] = c
    return out


def message(kind: str, a: str, b: str) -> str:
    reason = {"spelling": "differ only in case, whitespace or punctuation",
              "typo": "differ in a few letters"}[kind]
    return (f"two AI calls over the same columns {reason}, so the model would answer each: {a!r} and {b!r}. "
            f"Write the call the same way each time to ask the model once")
