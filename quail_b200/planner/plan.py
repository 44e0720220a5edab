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
    # what the physical section shows: the table alias an AI node reads, its prompt, its
    # selectivity (and whether it was assumed), a scan's token counts (planner/explain.py)
    info: dict = field(default_factory=dict)


@dataclass
class Plan:
    root: PlanNode
    settings: dict = field(default_factory=dict)
    envelope: dict = field(default_factory=dict)

    def nodes(self):
        out, stack = [], [self.root]
        while stack:
            n = stack.pop()
            out.append(n)
            stack.extend(reversed(n.children))
        return out

    def explain(self, verbose: bool = False) -> str:
        """The logical plan, then the physical plan with the planner's estimates."""
        from quail_b200.planner.explain import render
        return render(self, verbose=verbose)

    def logical(self, verbose: bool = False) -> str:
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
        """The physical plan's measured side after a run (rows, pass share, time, fresh tokens per
        model region), then the run's totals."""
        from quail_b200.planner.explain import render_measured
        return render_measured(self, report)

    def measured_totals(self, report: dict) -> str:
        keys = ("wall_s", "boot_s", "fresh_tokens", "cached_tokens", "evaluated_documents", "passes", "asked",
                "output_rows", "stopped_early", "peak_gib", "usd_per_query")
        return "totals: " + ", ".join(f"{k}={_short(report.get(k))}" for k in keys if k in report)


def _short(v):
    return f"{v:.4g}" if isinstance(v, float) else v


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


def _options_of(call) -> dict:
    """A call's options object: its second positional argument or its named `options`."""
    from quail_b200.sql.executor import literal_value
    args = [a for a in call.get("args", []) if isinstance(a, dict) and a.get("type") != "named_arg"]
    named = {a["name"].lower(): a["value"] for a in call.get("args", [])
             if isinstance(a, dict) and a.get("type") == "named_arg"}
    node = args[1] if len(args) > 1 else named.get("options")
    if node is None:
        return {}
    try:
        v = literal_value(node)
    except Exception:  # noqa: BLE001 - a non-literal option prices at the defaults
        return {}
    return v if isinstance(v, dict) else {}


def _selectivity(call) -> float:
    """The share of rows an AI filter keeps: its options' 'selectivity', else one half."""
    v = _options_of(call).get("selectivity")
    if isinstance(v, (int, float)):
        return min(max(float(v), 0.0), 1.0)
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
                                chunk_tokens=session.config.chunk_tokens,
                                registry=getattr(session, "registry", None))
    settings = {"model": session.config.model, "device": session.config.device, "gpus": session.config.gpus,
                "chunk_tokens": budgets.chunk_tokens, "compute_knee": budgets.compute_knee()}
    node = tree["query"] if tree.get("type") == "explain" else tree
    plan = Plan(root=_plan_select(node, session, budgets), settings=settings)
    plan.envelope = _envelope(session, budgets)
    return plan


def _envelope(session, budgets) -> dict:
    """The physical plan's header: backend, model, GPUs, memory budgets, architecture, kernels."""
    cfg = session.model_cfg
    cpu = session.config.device == "cpu"
    out = {"backend": "quail_b200", "model": session.config.model, "gpus": max(session.config.gpus, 1),
           "chunk_tokens": budgets.chunk_tokens, "kv": "fp32" if cpu else "bf16"}
    if cfg is None:
        return out
    try:
        page = 128 if session.config.device != "cpu" else 16
        out["admission_tokens"] = budgets.arena_pages(page) * page
    except Exception:  # noqa: BLE001 - a budget that does not fit is the executor's refusal, not explain's
        out["admission_tokens"] = None
    out["architecture"] = f"{cfg.arch} ({cfg.layers} layers)"
    weights = "nvfp4" if getattr(cfg, "mlp_fp4", False) else ("fp8" if getattr(cfg, "fp8", False) else "bf16")
    out["weights"] = weights
    gemm = {"fp8": "MX fp8 tcgen05 GEMM (1x32 UE8M0 activation scales)", "bf16": "bf16 tcgen05 GEMM",
            "nvfp4": "NVFP4 tcgen05 GEMM (attention fp8)"}[weights]
    attn = ("small-tile paged attention (head_dim %d)" % cfg.head_dim if cfg.is_hybrid or cfg.head_dim != 128
            else "persistent tcgen05 attention (TMEM accumulators)")
    out["kernels"] = f"linear layers: {gemm}; attention: {attn}"
    if cpu:
        out["kernels"] = "the fp32 statement of the model on the CPU (no GPU kernels)"
    elif cfg.is_hybrid:
        out["kernels"] += "; token mixers: " + ("gated delta rule (chunked)" if cfg.arch != "lfm2"
                                                 else "short convolution")
    return out


def _doc_column(call):
    """The column a call reads as its document (a plain column or PROMPT's one argument), or None."""
    args = [a for a in call.get("args", []) if isinstance(a, dict) and a.get("type") != "named_arg"]
    if not args:
        return None
    d = args[0]
    if d.get("type") == "call" and d.get("name") == "PROMPT" and len(d.get("args", [])) == 2:
        d = d["args"][1]
    return d.get("name") if d.get("type") == "column" else None


def _mean_doc_tokens(call, ref, session, default: float = 300.0, cache: dict | None = None) -> float:
    """Mean document length in tokens from a sample of the scanned column: token-id lists by
    their length, text at about 4 characters per token; `default` when it cannot tell.
    `cache` keeps one sample per (table, column) for the whole plan."""
    return _column_mean_tokens(ref, _doc_column(call), session, default, cache)


def _column_mean_tokens(ref, col, session, default: float = 300.0, cache: dict | None = None) -> float:
    if col is None or ref is None or ref.get("type") != "table":
        return default
    key = (ref["name"].lower(), col.lower())
    if cache is not None and key in cache:
        return cache[key]
    value = _sample_mean_tokens(ref, col, session, default)
    if cache is not None:
        cache[key] = value
    return value


def _sample_mean_tokens(ref, col, session, default: float) -> float:
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
    cache: dict = {}
    gpus = max(session.config.gpus, 1)
    tail_tokens = 60.0
    # a document-isolated model prefills its system turn with every document (no shared prefix KV)
    block_tokens = 48.0 if getattr(getattr(session, "model_cfg", None), "bidirectional", False) else 0.0
    scans = {}
    if node.get("from"):
        ref = node["from"][0]
        rows = _rows_of(ref, session)
        cur = PlanNode("quail.scan", ref.get("name", "subquery"), rows=rows, info=_scan_info(ref))
        scans[cur.info["alias"].lower()] = cur
        for j in node.get("joins", []):
            right = PlanNode("quail.scan", j["table"].get("name", "subquery"), rows=_rows_of(j["table"], session),
                             info=_scan_info(j["table"]))
            scans[right.info["alias"].lower()] = right
            kind = "AiJoin" if has_model_call(j.get("on")) else "HashJoin"
            r2 = right.rows
            left_rows = rows
            rows = rows * r2 if rows is not None and r2 is not None and kind == "AiJoin" else rows
            detail, secs, jinfo = j["kind"], None, {"join": j["kind"]}
            if kind == "AiJoin":
                detail, secs = _ai_join(j, ref, left_rows, r2, session, budgets, cache, tail_tokens)
                call = next(n for n in walk(j.get("on")) if is_model_call(n))
                jinfo = {**_call_info(call, rows, None), "join": j["kind"], "detail": detail}
            cur = PlanNode(kind, detail, rows=rows, seconds=secs, children=[cur, right], info=jinfo)
    base_ref = node["from"][0] if node.get("from") and not node.get("joins") else None
    for c in conjuncts(node.get("where")):
        if not has_model_call(c):
            cur = PlanNode("Filter", _expr_text(c), rows=rows, children=[cur] if cur else [])
    # AI filters in the order the executor asks them (planner.search.order_filters)
    ai_conj = [c for c in conjuncts(node.get("where")) if has_model_call(c)]
    ai_conj = _ordered_filters(ai_conj, session)
    doc_read = set()
    for c in ai_conj:
        for n in walk(c):
            if is_model_call(n):
                secs = None
                mean_doc_tokens = _mean_doc_tokens(n, base_ref, session, cache=cache)
                if rows is not None:
                    first = _doc_column(n) not in doc_read
                    tokens = rows * ((mean_doc_tokens + block_tokens if first else 0.0) + tail_tokens)
                    secs = budgets.pass_seconds(int(tokens), mean_doc_tokens / 2) / gpus
                doc_read.add(_doc_column(n))
                cur = PlanNode(NODE_OF[n["name"]], _expr_text(n)[:80], rows=rows, seconds=secs,
                               children=[cur] if cur else [], info=_call_info(n, rows, base_ref))
                _note_scan(scans, cur.info, rows, mean_doc_tokens)
                rows = rows * _selectivity(n) if rows is not None else None
    for it in node["items"]:
        for n in walk(it["expr"]):
            if is_model_call(n):
                secs = None
                mean_doc_tokens = _mean_doc_tokens(n, base_ref, session, cache=cache)
                if rows is not None:
                    # a document no earlier model call read is prefilled here
                    fresh = tail_tokens + (0.0 if _doc_column(n) in doc_read else mean_doc_tokens + block_tokens)
                    doc_read.add(_doc_column(n))
                    secs = budgets.pass_seconds(int(rows * fresh), mean_doc_tokens)
                    steps = _decode_tokens(n)
                    if steps:
                        # greedy decode: one token per row per step over the row's context
                        secs += steps * budgets.pass_seconds(max(int(rows), 1), mean_doc_tokens + steps / 2)
                    secs /= gpus
                cur = PlanNode(NODE_OF[n["name"]], _expr_text(n)[:80], rows=rows, seconds=secs,
                               children=[cur] if cur else [], info=_call_info(n, rows, base_ref))
                _note_scan(scans, cur.info, rows, mean_doc_tokens)
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


def _scan_info(ref) -> dict:
    name = ref.get("name", "subquery")
    return {"table": name, "alias": ref.get("alias") or name}


def _note_scan(scans: dict, info: dict, rows, mean_doc_tokens: float) -> None:
    """The scan an AI node reads gets its document token counts (first reader's column)."""
    scan = scans.get((info.get("alias") or "").lower()) or (next(iter(scans.values())) if len(scans) == 1 else None)
    if scan is None or "mean_document_tokens" in scan.info:
        return
    scan.info["mean_document_tokens"] = mean_doc_tokens
    if scan.rows is not None:
        scan.info["tokens"] = scan.rows * mean_doc_tokens


def _call_info(call, rows, base_ref) -> dict:
    """What the physical section shows of an AI node: the alias of the table it reads, its
    prompt (the PROMPT template, an instruction or the questions), its input rows and, for a
    filter, its selectivity and whether the planner assumed it."""
    from quail_b200.sql.executor import literal_value
    args = [a for a in call.get("args", []) if isinstance(a, dict) and a.get("type") != "named_arg"]
    info = {"kind": call["name"], "rows_in": rows}
    d = args[0] if args else {}
    cols = [n for n in walk(d) if n.get("type") == "column"]
    alias = next((c.get("table") for c in cols if c.get("table")), None)
    if alias is None and base_ref is not None:
        alias = base_ref.get("alias") or base_ref.get("name")
    info["alias"] = alias or ""
    prompt = None
    if d.get("type") == "call" and d.get("name") == "PROMPT" and d.get("args"):
        try:
            prompt = literal_value(d["args"][0])
        except Exception:  # noqa: BLE001 - a computed template shows as written
            prompt = None
    try:
        second = literal_value(args[1]) if len(args) > 1 else None
    except Exception:  # noqa: BLE001 - options that are not constants
        second = None
    if call["name"] in ("AI.IF", "AI_FILTER"):
        v = _options_of(call).get("selectivity")
        info["selectivity"] = _selectivity(call)
        info["assumed"] = not isinstance(v, (int, float))
    elif call["name"] == "AI.CLASSIFY" and isinstance(second, list):
        info["labels"] = len(second)
    elif call["name"] == "AI.MAP":
        prompt = prompt or (second if isinstance(second, str) else None)
        info["max_tokens"] = _decode_tokens(call)
    elif call["name"] in ("AI.EXTRACT", "AI.EXTRACT_SPAN"):
        qs = second if isinstance(second, (list, dict)) else [second]
        info["questions"] = len(qs)
        prompt = prompt or (", ".join(str(q) for q in (qs.values() if isinstance(qs, dict) else qs)))
    info["prompt"] = prompt if prompt is not None else "{0}"
    return info


def _ordered_filters(ai_conj: list, session) -> list:
    """WHERE conjuncts with model calls: AI.IF ones in the executor's cost order, then the rest."""
    from quail_b200.planner.search import doc_tokens, order_filters
    from quail_b200.sql.executor import bind_call
    filters, others = [], []
    for c in ai_conj:
        inner = c["args"][0] if c.get("type") == "call" and c.get("name") == "HINT" else c
        (filters if is_model_call(inner) and inner["name"] in ("AI.IF", "AI_FILTER") else others).append(c)
    if len(filters) < 2:
        return filters + others
    try:
        from quail_b200.api import prompts as P
        model = P.prompt_model(session.model_cfg) if session.model_cfg is not None else P.PromptModel()
        bound = [bind_call(c["args"][0] if c.get("name") == "HINT" else c, model.turn, model) for c in filters]
        order = order_filters([doc_tokens(b.tail) for b in bound],
                              [b.selectivity if b.selectivity is not None else 0.5 for b in bound])
    except Exception:  # noqa: BLE001 - a call the binder refuses keeps the written order
        return filters + others
    return [filters[i] for i in order] + others


def _ai_join(j, left_ref, left_rows, right_rows, session, budgets, cache, tail_tokens):
    """Detail and cost of an AI join: its anchor side (planner.search) and the pair prefill."""
    on = j.get("on")
    call = next((n for n in walk(on) if is_model_call(n)), None)
    if call is None:
        return j["kind"], None
    args = [a for a in call.get("args", []) if isinstance(a, dict) and a.get("type") != "named_arg"]
    prompt = args[0] if args else None
    if not (prompt and prompt.get("type") == "call" and prompt.get("name") == "PROMPT"
            and len(prompt.get("args", [])) == 3):
        return j["kind"], None
    a, b = prompt["args"][1], prompt["args"][2]
    right_ref = j["table"]

    def side_of(e):
        q = e.get("table") if e.get("type") == "column" else None
        if q is not None and q.lower() in ((right_ref.get("alias") or right_ref.get("name") or "").lower(),):
            return "R"
        return "L"
    lexpr, rexpr = (a, b) if side_of(a) == "L" else (b, a)
    lm = _column_mean_tokens(left_ref, lexpr.get("name") if lexpr.get("type") == "column" else None, session,
                             cache=cache)
    rm = _column_mean_tokens(right_ref, rexpr.get("name") if rexpr.get("type") == "column" else None, session,
                             cache=cache)
    if left_rows is None or right_rows is None:
        return f"{j['kind']}, anchor by cost at run time", None
    pairs = left_rows * right_rows
    asked = _options_of(call).get("anchor")
    cost_l = left_rows * lm + pairs * (rm + tail_tokens)
    cost_r = right_rows * rm + pairs * (lm + tail_tokens)
    if asked is not None:
        anchor = "left" if str(asked).lower() in ("left", "l", "0", "first") else "right"
    else:
        anchor = "left" if cost_l <= cost_r else "right"
    tokens = cost_l if anchor == "left" else cost_r
    secs = budgets.pass_seconds(int(tokens), (lm + rm) / 2) / max(session.config.gpus, 1)
    expr = _expr_text(lexpr if anchor == "left" else rexpr)
    return f"{j['kind']}, anchor={anchor} ({expr}), pairs={pairs:.0f}", secs
