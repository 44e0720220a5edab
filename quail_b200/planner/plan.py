"""Logical and physical plan of a query, with roofline estimates, as explain text.

The reference's planner turns a region into physical nodes
(quail.scan / ai_filter / ai_score / ai_classify / ai_map / filter / limit /
hash_join ..., crates/quail-planner/src/physical/nodes.rs:168-349) and prints
estimated times per node (explain.rs). This planner derives the same node
sequence from the syntax tree in the order the executor runs it (relational
conjuncts first, the guarded AI.IF chain, then projection calls) and prices
each model node with the roofline of `Budgets.pass_seconds`: prefill of the
document and question tokens, plus one pass per generated token for AI.MAP /
AI.EXTRACT; an AI filter keeps its options' 'selectivity' share of the rows
(one half without one).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from quail_b200.sql.executor import conjuncts, has_model_call, is_model_call, walk

NODE_OF = {"AI.IF": "AiFilter", "AI_FILTER": "AiFilter", "AI.SCORE": "AiScore", "AI.CLASSIFY": "AiClassify",
           "AI.MAP": "AiMap", "AI.EXTRACT": "AiExtract", "AI.EXTRACT_SPAN": "AiExtract",
           "AI.SAE_FEATURES": "AiSaeFeatures"}


@dataclass
class PlanNode:
    name: str
    detail: str = ""
    rows: float | None = None
    seconds: float | None = None
    children: list = field(default_factory=list)


@dataclass
class Plan:
    root: PlanNode
    settings: dict = field(default_factory=dict)

    def nodes(self):
        out, stack = [], [self.root]
        while stack:
            n = stack.pop()
            out.append(n)
            stack.extend(reversed(n.children))
        return out

    def explain(self, verbose: bool = False) -> str:
        lines = []

        def rec(n: PlanNode, depth: int):
            est = []
            if n.rows is not None:
                est.append(f"rows={n.rows:.0f}")
            if n.seconds is not None:
                est.append(f"est={n.seconds * 1e3:.2f}ms")
            lines.append("  " * depth + n.name + (f": {n.detail}" if n.detail else "")
                         + (f"  [{', '.join(est)}]" if est else ""))
            for c in n.children:
                rec(c, depth + 1)

        rec(self.root, 0)
        if verbose and self.settings:
            lines.append("settings: " + ", ".join(f"{k}={v}" for k, v in sorted(self.settings.items())))
        return "\n".join(lines)

    def explain_measured(self, report: dict) -> str:
        keys = ("wall_s", "boot_s", "fresh_tokens", "evaluated_documents", "passes", "asked", "output_rows")
        return "measured: " + ", ".join(f"{k}={report.get(k)}" for k in keys if k in report)


def _expr_text(e) -> str:
    t = e.get("type")
    if t == "column":
        return (e["table"] + "." if e.get("table") else "") + e["name"]
    if t == "literal":
        return repr(e["value"])
    if t == "call":
        return e["name"] + "(" + ", ".join(_expr_text(a) for a in e.get("args", []) if isinstance(a, dict)) + ")"
    if t == "binary":
        return f"{_expr_text(e['left'])} {e['op']} {_expr_text(e['right'])}"
    if t == "array":
        return "[" + ", ".join(_expr_text(i) for i in e.get("items", [])) + "]"
    if t == "object":
        return "{" + ", ".join(f"{k!r}: {_expr_text(v)}" for k, v in e.get("items", [])) + "}"
    return t


def _selectivity(call) -> float:
    """The share of rows an AI filter keeps: its options' 'selectivity', else one half."""
    from quail_b200.sql.executor import literal_value
    args = [a for a in call.get("args", []) if isinstance(a, dict) and a.get("type") != "named_arg"]
    if len(args) > 1:
        try:
            v = literal_value(args[1])
            if isinstance(v, dict) and isinstance(v.get("selectivity"), (int, float)):
                return min(max(float(v["selectivity"]), 0.0), 1.0)
        except Exception:  # noqa: BLE001 - a non-literal option prices at the default
            pass
    return 0.5


def _decode_tokens(call) -> int:
    """Tokens a decoding call generates per row at most (AI.MAP's max_tokens, AI.EXTRACT's 64 per question)."""
    from quail_b200.sql.executor import MAP_DEFAULT_TOKENS, literal_value
    args = [a for a in call.get("args", []) if isinstance(a, dict) and a.get("type") != "named_arg"]
    if call["name"] == "AI.MAP":
        v = literal_value(args[2]) if len(args) > 2 else MAP_DEFAULT_TOKENS
        return int(v) if isinstance(v, int) else MAP_DEFAULT_TOKENS
    if call["name"] in ("AI.EXTRACT", "AI.EXTRACT_SPAN"):
        qs = literal_value(args[1]) if len(args) > 1 else []
        return 64 * (1 if isinstance(qs, str) else max(len(qs), 1))
    return 0


def plan_query(tree: dict, session) -> Plan:
    from quail_b200.planner.budgets import Budgets
    cfg = session.model_cfg
    budgets = Budgets.for_model(cfg, session.config.device, gpus=session.config.gpus,
                                chunk_tokens=session.config.chunk_tokens)
    settings = {"model": session.config.model, "device": session.config.device, "gpus": session.config.gpus,
                "chunk_tokens": budgets.chunk_tokens, "compute_knee": budgets.compute_knee()}
    node = tree["query"] if tree.get("type") == "explain" else tree
    return Plan(root=_plan_select(node, session, budgets), settings=settings)


def _doc_column(call):
    """The column a call reads as its document (a plain column or PROMPT's one argument), or None."""
    args = [a for a in call.get("args", []) if isinstance(a, dict) and a.get("type") != "named_arg"]
    if not args:
        return None
    d = args[0]
    if d.get("type") == "call" and d.get("name") == "PROMPT" and len(d.get("args", [])) == 2:
        d = d["args"][1]
    return d.get("name") if d.get("type") == "column" else None


def _mean_doc_tokens(call, ref, session, default: float = 300.0) -> float:
    """Mean document length in tokens from a sample of the scanned column: token-id lists by
    their length, text at about 4 characters per token; `default` when it cannot tell."""
    col = _doc_column(call)
    if col is None or ref is None or ref.get("type") != "table":
        return default
    try:
        from quail_b200.catalog.providers import ScanRequest
        for k, p in session.catalog.items():
            if k.lower() != ref["name"].lower():
                continue
            name = next((c for c in p.columns if c.lower() == col.lower()), None)
            if name is None:
                return default
            vals = p.scan(ScanRequest(columns=(name,), limit=256)).read_all().column(0).to_pylist()
            lens = [len(v) / (4.0 if isinstance(v, str) else 1.0) for v in vals if v is not None]
            return max(sum(lens) / len(lens), 1.0) if lens else default
    except Exception:  # noqa: BLE001 - statistics are best effort
        return default
    return default


def _rows_of(ref, session) -> float | None:
    if ref.get("type") != "table":
        return None
    for k, p in session.catalog.items():
        if k.lower() == ref["name"].lower():
            try:
                return float(p.statistics().num_rows)
            except Exception:  # noqa: BLE001 - statistics are best effort
                return None
    return None


def _plan_select(node, session, budgets) -> PlanNode:
    if node.get("type") == "union":
        return PlanNode("Union", "ALL" if node["all"] else "DISTINCT",
                        children=[_plan_select(node["left"], session, budgets),
                                  _plan_select(node["right"], session, budgets)])
    if node.get("type") != "select":
        return PlanNode(node.get("type", "?"))
    cur = None
    rows = None
    if node.get("from"):
        ref = node["from"][0]
        rows = _rows_of(ref, session)
        cur = PlanNode("quail.scan", ref.get("name", "subquery"), rows=rows)
        for j in node.get("joins", []):
            right = PlanNode("quail.scan", j["table"].get("name", "subquery"), rows=_rows_of(j["table"], session))
            kind = "AiJoin" if has_model_call(j.get("on")) else "HashJoin"
            r2 = right.rows
            rows = rows * r2 if rows is not None and r2 is not None and kind == "AiJoin" else rows
            cur = PlanNode(kind, j["kind"], rows=rows, children=[cur, right])
    base_ref = node["from"][0] if node.get("from") and not node.get("joins") else None
    tail_tokens = 60.0
    for c in conjuncts(node.get("where")):
        if not has_model_call(c):
            cur = PlanNode("Filter", _expr_text(c), rows=rows, children=[cur] if cur else [])
    for c in conjuncts(node.get("where")):
        for n in walk(c):
            if is_model_call(n):
                secs = None
                mean_doc_tokens = _mean_doc_tokens(n, base_ref, session)
                if rows is not None:
                    tokens = rows * (mean_doc_tokens + tail_tokens)
                    secs = budgets.pass_seconds(int(tokens), mean_doc_tokens / 2) / max(session.config.gpus, 1)
                cur = PlanNode(NODE_OF[n["name"]], _expr_text(n)[:80], rows=rows, seconds=secs,
                               children=[cur] if cur else [])
                rows = rows * _selectivity(n) if rows is not None else None
    for it in node["items"]:
        for n in walk(it["expr"]):
            if is_model_call(n):
                secs = None
                mean_doc_tokens = _mean_doc_tokens(n, base_ref, session)
                if rows is not None:
                    secs = budgets.pass_seconds(int(rows * tail_tokens), mean_doc_tokens)
                    steps = _decode_tokens(n)
                    if steps:
                        # greedy decode: one token per row per step over the row's context
                        secs += steps * budgets.pass_seconds(max(int(rows), 1), mean_doc_tokens + steps / 2)
                    secs /= max(session.config.gpus, 1)
                cur = PlanNode(NODE_OF[n["name"]], _expr_text(n)[:80], rows=rows, seconds=secs,
                               children=[cur] if cur else [])
    if node.get("group_by") is not None:
        cur = PlanNode("Aggregate", ", ".join(_expr_text(g) for g in node["group_by"]), children=[cur] if cur else [])
    cur = PlanNode("Projection", ", ".join(it.get("alias") or _expr_text(it["expr"]) for it in node["items"])[:120],
                   rows=rows, children=[cur] if cur else [])
    if node.get("order_by"):
        cur = PlanNode("Sort", ", ".join(_expr_text(o["expr"]) + (" DESC" if o["desc"] else "")
                                         for o in node["order_by"]), children=[cur])
    if node.get("limit") is not None:
        cur = PlanNode("Limit", _expr_text(node["limit"]), children=[cur])
    return cur
