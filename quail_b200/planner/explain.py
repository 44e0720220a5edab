"""The text of `explain()`: the logical plan, then the physical plan with estimates.

Layout (the reference's explain text, crates/quail-planner/src/explain.rs, kept
alike so a reader of one reads the other):

    logical:
      <the plan tree, one operator per line>

    physical: backend=quail_b200, model=<model>, gpus=<n>
      KV=<dtype>, chunk budget=<tokens> tokens, admission budget=<tokens> tokens
      architecture=<arch> (<layers> layers), weights=<dtype>
      kernels: <the kernels the model's layers run>

                                   est. rows   est. pass   est. time
      AiFilter: r                        0.4                 1.09 ms
        predicate 1  PROMPT('Is the review positive? {0}')     2     50%*
        Scan reviews as r                  2
          tokens=10, mean_document_tokens=5
      * no selectivity was given; the planner assumes 50%
      est. time is each node's work alone; ...

After a run, `render_measured` gives the measured side: per model region the
rows in and out, the share that passed, its time and its fresh tokens, then
the run's totals. The physical section lists model nodes, scans, plain
filters, joins, aggregates and limits; projections and sorts stay in the
logical section. The rendering is this build's own.
"""

from __future__ import annotations

PROMPT_CHARS = 32
COLS = ("est. rows", "est. pass", "est. time")
MEASURED_COLS = ("rows in", "rows", "pass", "time", "fresh tokens")
# a measured region's other counts, on the line below it
DETAIL = ("evaluated_documents", "cached_tokens", "kv_hits", "kv_misses", "kv_removals", "kv_recomputations",
          "chunks", "peak_gpu_bytes")
AI_NODES = ("AiFilter", "AiScore", "AiClassify", "AiMap", "AiExtract", "AiSaeFeatures")


def _rows(v) -> str:
    if v is None:
        return ""
    return f"{v:.2g}" if v < 10 else f"{v:,.0f}"


def _pct(p: float) -> str:
    return f"{p * 100:.3g}%"


def _time(sec) -> str:
    if sec is None:
        return ""
    if sec >= 1.0:
        return f"{sec:.3g} s"
    ms = sec * 1e3
    return f"{ms:.3g} ms" if ms < 100 else f"{ms:.0f} ms"


def _prompt(text: str) -> str:
    t = text.encode("unicode_escape").decode("ascii").replace("'", "\\'")
    if len(t) > PROMPT_CHARS:
        t = t[:PROMPT_CHARS] + "…"
    return f"PROMPT('{t}')"


def _lines(node, depth: int, out: list, state: dict) -> None:
    """(indent, label, cells) rows of the physical tree under `node`."""
    name, info = node.name, node.info
    pad = "  " * depth
    if name in ("Projection", "Sort"):
        for c in node.children:
            _lines(c, depth, out, state)
        return
    if name == "quail.scan":
        alias = info.get("alias", node.detail)
        label = f"Scan {info.get('table', node.detail)}" + (f" as {alias}" if alias != info.get("table") else "")
        out.append((pad + label, [_rows(node.rows), "", ""]))
        if "tokens" in info:
            out.append((pad + f"  tokens={info['tokens']:,.0f}, "
                        f"mean_document_tokens={info['mean_document_tokens']:.3g}", None))
        return
    if name in AI_NODES:
        label = f"{name}: {info.get('alias', '')}".rstrip(": ")
        out_rows = node.rows
        if name == "AiFilter" and node.rows is not None:
            out_rows = node.rows * info.get("selectivity", 0.5)
        out.append((pad + label, [_rows(out_rows), "", _time(node.seconds)]))
        if name == "AiFilter":
            state["predicates"] += 1
            sel = info.get("selectivity", 0.5)
            mark = "*" if info.get("assumed", True) else ""
            state["assumed"] |= bool(mark)
            out.append((pad + f"  predicate {state['predicates']}  {_prompt(info.get('prompt', '{0}'))}",
                        [_rows(info.get("rows_in")), _pct(sel) + mark, ""]))
        elif name == "AiClassify" and "labels" in info:
            out.append((pad + f"  labels={info['labels']}  {_prompt(info.get('prompt', '{0}'))}", None))
        elif name == "AiMap":
            out.append((pad + f"  max_tokens={info.get('max_tokens')}  {_prompt(info.get('prompt', '{0}'))}", None))
        elif name == "AiExtract":
            out.append((pad + f"  questions={info.get('questions')}  {_prompt(info.get('prompt', '{0}'))}", None))
        else:
            out.append((pad + f"  {_prompt(info.get('prompt', '{0}'))}", None))
    elif name == "AiJoin":
        out.append((pad + f"AiJoin: {info.get('detail', node.detail)}", [_rows(node.rows), "", _time(node.seconds)]))
        out.append((pad + f"  join {info.get('join', '')} ({info.get('alias', '')})  "
                    f"{_prompt(info.get('prompt', '{0}'))}", [_rows(node.rows), "", ""]))
    elif name == "HashJoin":
        out.append((pad + f"HashJoin: {node.detail}", [_rows(node.rows), "", ""]))
    else:
        out.append((pad + f"{name}: {node.detail}".rstrip(": "), [_rows(node.rows), "", _time(node.seconds)]))
    for c in node.children:
        _lines(c, depth + 1, out, state)


def _table(rows: list, cols: tuple, indent: str = "  ") -> list:
    width = max([len(r[0]) for r in rows] + [20]) + 4
    w = [max(len(c), 9) for c in cols]
    head = indent + " " * width + "   ".join(c.rjust(x) for c, x in zip(cols, w))
    out = [head.rstrip()]
    for label, cells in rows:
        if cells is None:
            out.append(indent + label)
            continue
        out.append((indent + label.ljust(width) + "   ".join(v.rjust(x) for v, x in zip(cells, w))).rstrip())
    return out


def render(plan, verbose: bool = False) -> str:
    lines = ["logical:"]
    lines += ["  " + ln for ln in plan.logical(verbose=False).splitlines()]
    env = getattr(plan, "envelope", {}) or {}
    lines.append("")
    lines.append(f"physical: backend={env.get('backend', 'quail_b200')}, model={env.get('model', '')}, "
                 f"gpus={env.get('gpus', 1)}")
    budget = f"  KV={env.get('kv', 'bf16')}, chunk budget={env.get('chunk_tokens', 0):,} tokens"
    if env.get("admission_tokens"):
        budget += f", admission budget={env['admission_tokens']:,} tokens"
    lines.append(budget)
    if "architecture" in env:
        lines.append(f"  architecture={env['architecture']}, weights={env['weights']}")
        lines.append(f"  kernels: {env['kernels']}")
    lines.append("")
    state = {"predicates": 0, "assumed": False}
    rows: list = []
    _lines(plan.root, 0, rows, state)
    lines += _table(rows, COLS)
    if state["assumed"]:
        lines.append("  * no selectivity was given; the planner assumes 50%")
    lines.append("  est. time is each node's work alone; node times do not add up to the plan estimate")
    lines.append("  because chunk packing shares forward passes across nodes")
    if verbose and plan.settings:
        lines.append("settings: " + ", ".join(f"{k}={v}" for k, v in sorted(plan.settings.items())))
    return "\n".join(lines)


def render_measured(plan, report: dict) -> str:
    """Per model region: rows in and out, pass share, time and fresh tokens; then totals."""
    rows = []
    for node, m in report.get("node_metrics", {}).items():
        if node == "output":
            continue
        rin, rout = m.get("input_rows", 0), m.get("output_rows", 0)
        share = _pct(rout / rin) if rin and "filter" in node else ""
        rows.append((node, [f"{rin:,}", f"{rout:,}", share, _time(m.get("wall_s")),
                            f"{m.get('fresh_tokens', 0):,}"]))
        detail = ", ".join(f"{k}={m[k]:,}" for k in DETAIL if m.get(k))
        if detail:
            rows.append(("  " + detail, None))
    out = ["measured:"]
    if rows:
        out += _table(rows, MEASURED_COLS)
    out.append(plan.measured_totals(report))
    return "\n".join(out)
