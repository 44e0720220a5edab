"""Choices the planner makes by cost: the order of AI filters and the anchor of an AI join.

Both use token counts as the cost of model work (a prefill pass's time is
close to linear in its fresh tokens at these sizes, see planner/budgets.py):

- filter order: for independent filters applied as a guarded chain, asking
  them in increasing order of cost / (1 - selectivity) minimizes the
  expected cost (each filter's cost is paid only by the rows the earlier ones
  kept); a filter's cost is its question's tokens (the document is read once,
  by the first question, whatever the order);
- join anchor: with one side's documents prefilled once and every pair
  computing the other document and the question, the anchor is the side
  whose choice leaves fewer fresh tokens: sum of the anchor side's distinct
  documents + sum over pairs of the other side's document.

Reference: crates/quail-planner/src/search.rs:408 (operator order) and
:891 (join anchors), cost/pricing.rs.
"""

from __future__ import annotations


def doc_tokens(text) -> float:
    """A document's tokens without a tokenizer: about four characters per token."""
    if text is None:
        return 0.0
    if isinstance(text, (list, tuple)):
        return float(len(text))
    return max(len(str(text)) / 4.0, 1.0)


def join_costs(left: list, right: list) -> tuple[float, float]:
    """Fresh tokens of the pair questions with the left or the right side as the anchor."""
    n = len(left)
    lt = [doc_tokens(x) for x in left]
    rt = [doc_tokens(x) for x in right]
    anchor_left = sum(doc_tokens(x) for x in set(left)) + sum(rt[:n])
    anchor_right = sum(doc_tokens(x) for x in set(right)) + sum(lt[:n])
    return anchor_left, anchor_right


def choose_anchor(left: list, right: list, asked: str | None = None) -> str:
    """'L' or 'R': the join anchor, by cost unless the query names one ({'anchor': 'left'|'right'})."""
    if asked is not None:
        a = str(asked).lower()
        if a in ("left", "l", "0", "first"):
            return "L"
        if a in ("right", "r", "1", "second"):
            return "R"
    cl, cr = join_costs(left, right)
    return "L" if cl <= cr else "R"


def order_filters(costs: list[float], selectivities: list[float]) -> list[int]:
    """Indices of the filters in the order that minimizes the expected cost of the chain."""
    def rank(i):
        keep = min(max(selectivities[i], 0.0), 0.999)
        return costs[i] / (1.0 - keep)
    return sorted(range(len(costs)), key=rank)
