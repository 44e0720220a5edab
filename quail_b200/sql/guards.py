"""Demand rules: on which rows each model call must be asked.

A model call inside an expression is only worth asking where its value can
reach the result. This module walks an expression with the condition under
which the walk reaches each node (a *guard*) and records, for every model
call, the disjunction of the guards it is reached under:

- ``CASE WHEN c THEN a ELSE b END``: ``a`` under ``c``, ``b`` under ``NOT c``
  (each later WHEN under the earlier ones being false);
- ``x AND y``: ``y`` only where ``x`` is not FALSE; ``x OR y``: ``y`` only
  where ``x`` is not TRUE (this is the OR-guard: ``col > 5 OR AI.IF(...)``
  asks the model only on the rows the plain side leaves open);
- ``IFF(c, a, b)``, ``COALESCE(a, b)``, ``NULLIF`` the same way.

A guard is a small three-valued boolean formula, kept as plain JSON-able
dicts so it can travel to worker processes with the region:

  {"op": "true"} | {"op": "false"}
  {"op": "const", "v": [True | False | None per row]}      (a condition without model calls)
  {"op": "ai", "call": key, "cmp": None | "=" | "<>" | "<" | ..., "rhs": {"v": [...]} | {"lit": x}}
  {"op": "not" | "is_true" | "not_false" | "not_true" | "is_null", "a": g}
  {"op": "and" | "or", "a": g, "b": g}

An ``ai`` leaf reads the SQL value of another call of the same region (the
region's chain asks that call first); leaves that name calls answered by an
earlier region are folded into ``const`` leaves before the region starts
(`fold`). The reference states the same rules as DataFusion logical rules:
crates/quail-datafusion/src/rules/guards.rs:1-17 (CASE guards),
rules/or_guards.rs (OR guards) and rules/derive/demand.rs.
"""

from __future__ import annotations

import json

TRUE = {"op": "true"}
FALSE = {"op": "false"}

_CMP = {"=", "<>", "!=", "<", "<=", ">", ">="}
_FLIP = {"<": ">", "<=": ">=", ">": "<", ">=": "<=", "=": "=", "<>": "<>", "!=": "!="}


# ---------------------------------------------------------------- construction with simplification

def g_not(a):
    if a["op"] == "true":
        return FALSE
    if a["op"] == "false":
        return TRUE
    return {"op": "not", "a": a}


def g_and(a, b):
    if a["op"] == "false" or b["op"] == "false":
        return FALSE
    if a["op"] == "true":
        return b
    if b["op"] == "true":
        return a
    return {"op": "and", "a": a, "b": b}


def g_or(a, b):
    if a["op"] == "true" or b["op"] == "true":
        return TRUE
    if a["op"] == "false":
        return b
    if b["op"] == "false":
        return a
    return {"op": "or", "a": a, "b": b}


def _test(op, a):
    if a["op"] in ("true", "false"):
        value = a["op"] == "true"
        return TRUE if {"is_true": value, "not_false": value, "not_true": not value,
                        "is_null": False}[op] else FALSE
    return {"op": op, "a": a}


def is_true(a):
    return _test("is_true", a)


def not_false(a):
    return _test("not_false", a)


def not_true(a):
    return _test("not_true", a)


def is_null(a):
    return _test("is_null", a)


# ---------------------------------------------------------------- evaluation

def _cmp(op, x, y):
    if x is None or y is None:
        return None
    try:
        if op == "=":
            return x == y
        if op in ("<>", "!="):
            return x != y
        if op == "<":
            return x < y
        if op == "<=":
            return x <= y
        if op == ">":
            return x > y
        if op == ">=":
            return x >= y
    except TypeError:
        return None
    raise ValueError(f"unknown comparison {op}")


def evaluate(g, row: int, values: dict):
    """The guard's three-valued truth on `row`, given the row's answers so far (call key -> SQL value)."""
    op = g["op"]
    if op == "true":
        return True
    if op == "false":
        return False
    if op == "const":
        return g["v"][row]
    if op == "ai":
        v = values.get(g["call"])
        if g.get("cmp") is None:
            return None if v is None else bool(v)
        rhs = g["rhs"]
        other = rhs["v"][row] if "v" in rhs else rhs.get("lit")
        return _cmp(g["cmp"], v, other)
    if op == "not":
        a = evaluate(g["a"], row, values)
        return None if a is None else not a
    if op == "and":
        a = evaluate(g["a"], row, values)
        if a is False:
            return False
        b = evaluate(g["b"], row, values)
        if b is False:
            return False
        return None if a is None or b is None else True
    if op == "or":
        a = evaluate(g["a"], row, values)
        if a is True:
            return True
        b = evaluate(g["b"], row, values)
        if b is True:
            return True
        return None if a is None or b is None else False
    a = evaluate(g["a"], row, values)
    if op == "is_true":
        return a is True
    if op == "not_false":
        return a is not False
    if op == "not_true":
        return a is not True
    if op == "is_null":
        return a is None
    raise ValueError(f"unknown guard {op}")


def _possible(g, row: int) -> set:
    """Every value the guard can take on `row` whatever the region's answers turn out to be."""
    op = g["op"]
    if op == "true":
        return {True}
    if op == "false":
        return {False}
    if op == "const":
        return {g["v"][row]}
    if op == "ai":
        return {True, False, None}
    if op in ("and", "or"):
        a, b = _possible(g["a"], row), _possible(g["b"], row)
        out = set()
        for x in a:
            for y in b:
                out.add(evaluate({"op": op, "a": _lit(x), "b": _lit(y)}, 0, {}))
        return out
    return {evaluate({"op": op, "a": _lit(x)}, 0, {}) for x in _possible(g["a"], row)}


def _lit(x):
    return {"op": "const", "v": [x]}


def may_ask(g, row: int) -> bool:
    """False only when no answer of the region can make the guard TRUE on `row`."""
    return True in _possible(g, row)


def asks(g, row: int, values: dict) -> bool:
    """A call is asked on a row exactly where its guard is TRUE."""
    return g is None or evaluate(g, row, values) is True


# ---------------------------------------------------------------- rewriting

def calls_of(g) -> set:
    """Keys of the calls an ``ai`` leaf of the guard reads."""
    if g is None:
        return set()
    if g["op"] == "ai":
        return {g["call"]}
    out = set()
    for k in ("a", "b"):
        if k in g:
            out |= calls_of(g[k])
    return out


def fold(g, known: dict, n: int):
    """Replace ``ai`` leaves of calls in `known` (key -> per-row SQL values) by const leaves."""
    if g is None:
        return None
    op = g["op"]
    if op == "ai":
        if g["call"] not in known:
            return g
        vals = known[g["call"]]
        return {"op": "const", "v": [evaluate(g, r, {g["call"]: vals[r]}) for r in range(n)]}
    if op in ("and", "or"):
        a, b = fold(g["a"], known, n), fold(g["b"], known, n)
        return g_and(a, b) if op == "and" else g_or(a, b)
    if op == "not":
        return g_not(fold(g["a"], known, n))
    if "a" in g:
        return _test(op, fold(g["a"], known, n))
    return g


def take(g, rows: list):
    """The guard restricted to `rows` (in that order): per-row leaves are re-indexed."""
    if g is None:
        return None
    op = g["op"]
    if op == "const":
        return {"op": "const", "v": [g["v"][r] for r in rows]}
    if op == "ai":
        out = dict(g)
        if "v" in g.get("rhs", {}):
            out["rhs"] = {"v": [g["rhs"]["v"][r] for r in rows]}
        return out
    out = {"op": op}
    for k in ("a", "b"):
        if k in g:
            out[k] = take(g[k], rows)
    return out


def signature(g, row: int) -> tuple:
    """The row's values of every per-row leaf: rows with equal documents and equal signatures
    are asked the same questions, so a region may answer them once."""
    if g is None:
        return ()
    op = g["op"]
    if op == "const":
        return (g["v"][row],)
    if op == "ai":
        rhs = g.get("rhs", {})
        return (rhs["v"][row],) if "v" in rhs else ()
    out = ()
    for k in ("a", "b"):
        if k in g:
            out += signature(g[k], row)
    return out


def describe(g) -> str:
    """A short human reading of a guard (explain output, transcripts)."""
    op = g["op"]
    if op in ("true", "false"):
        return op.upper()
    if op == "const":
        v = g["v"]
        return f"<column condition: {sum(1 for x in v if x is True)} of {len(v)} rows>"
    if op == "ai":
        name = _short(g["call"])
        if g.get("cmp") is None:
            return name
        rhs = g["rhs"]
        return f"{name} {g['cmp']} {rhs['lit']!r}" if "lit" in rhs else f"{name} {g['cmp']} <column>"
    if op in ("and", "or"):
        return f"({describe(g['a'])} {op.upper()} {describe(g['b'])})"
    if op == "not":
        return f"NOT {describe(g['a'])}"
    return f"{describe(g['a'])} {op.replace('_', ' ').upper()}"


def _short(key: str) -> str:
    try:
        node = json.loads(key)
        return node.get("name", "call")
    except (ValueError, AttributeError):
        return str(key)[:24]


# ---------------------------------------------------------------- the demand walk

class Demand:
    """Walks expressions and records each model call's guard.

    `ex` is the executor: it evaluates conditions without model calls over
    the relation (``const`` leaves) and names calls by their node key.
    After `visit`, `guards` maps call key -> (call node, guard).
    """

    def __init__(self, ex, rel, enabled: bool = True):
        self.ex = ex
        self.rel = rel
        self.enabled = enabled
        self.guards: dict = {}

    # conditions -> guards ------------------------------------------------
    def _const(self, node):
        from quail_b200.sql.executor import _as_array, _bool
        n = self.rel.num_rows
        v = self.ex.eval(node, self.rel)
        try:
            vals = _as_array(_bool(v), n).to_pylist()
        except Exception:  # noqa: BLE001 - not a boolean: the condition is not a guard
            return None
        return {"op": "const", "v": vals}

    def _values(self, node):
        from quail_b200.sql.executor import _as_array
        v = self.ex.eval(node, self.rel)
        return _as_array(v, self.rel.num_rows).to_pylist()

    def compile(self, node):
        """The three-valued formula of a condition, or None when it cannot be stated as one."""
        from quail_b200.sql.executor import has_model_call, is_model_call, literal_value, node_key
        if node is None:
            return None
        if not has_model_call(node):
            return self._const(node)
        t = node.get("type")
        if is_model_call(node):
            if node["name"] in ("AI.IF", "AI_FILTER"):
                return {"op": "ai", "call": node_key(node), "cmp": None}
            return None
        if t == "call" and node["name"] == "HINT":
            return self.compile(node["args"][0])
        if t == "binary" and node["op"] in ("AND", "OR"):
            a, b = self.compile(node["left"]), self.compile(node["right"])
            if a is None or b is None:
                return None
            return g_and(a, b) if node["op"] == "AND" else g_or(a, b)
        if t == "unary" and node["op"] == "NOT":
            a = self.compile(node["arg"])
            return None if a is None else g_not(a)
        if t == "binary" and node["op"] in _CMP:
            left, right, op = node["left"], node["right"], node["op"]
            if not is_model_call(left):
                left, right, op = right, left, _FLIP[op]
            if not is_model_call(left) or has_model_call(right):
                return None
            try:
                rhs = {"lit": literal_value(right)}
            except Exception:  # noqa: BLE001 - a column or an expression: per-row values
                rhs = {"v": self._values(right)}
            return {"op": "ai", "call": node_key(left), "cmp": op, "rhs": rhs}
        if t == "is_null":
            a = self._value_leaf(node["arg"])
            if a is None:
                return None
            g = is_null(a)
            return g_not(g) if node["negated"] else g
        if t == "is_bool":
            a = self.compile(node["arg"])
            if a is None:
                return None
            g = is_true(a) if node["value"] else _test("is_true", g_not(a))
            return g_not(g) if node["negated"] else g
        return None

    def _value_leaf(self, node):
        from quail_b200.sql.executor import has_model_call, is_model_call, node_key
        if is_model_call(node):
            return {"op": "ai", "call": node_key(node), "cmp": None}
        if not has_model_call(node):
            vals = self._values(node)
            return {"op": "const", "v": [None if v is None else True for v in vals]}
        return None

    # the walk ------------------------------------------------------------
    def visit(self, node, guard=TRUE):
        from quail_b200.sql.executor import has_model_call, is_model_call, node_key
        if guard["op"] == "false" or not isinstance(node, (dict, list)):
            return
        if isinstance(node, list):
            for x in node:
                self.visit(x, guard)
            return
        if not has_model_call(node):
            return
        if is_model_call(node):
            k = node_key(node)
            old = self.guards.get(k)
            self.guards[k] = (node, guard if old is None else g_or(old[1], guard))
            return
        if not self.enabled:
            for v in node.values():
                self.visit(v, guard)
            return
        t = node.get("type")
        if t == "case":
            self._case(node, guard)
        elif t == "binary" and node["op"] in ("AND", "OR"):
            self.visit(node["left"], guard)
            lg = self.compile(node["left"])
            if lg is None:
                self.visit(node["right"], guard)
            else:
                keep = not_false(lg) if node["op"] == "AND" else not_true(lg)
                self.visit(node["right"], g_and(guard, keep))
        elif t == "call" and node["name"] == "IFF" and len(node["args"]) == 3:
            c, a, b = node["args"]
            self.visit(c, guard)
            cg = self.compile(c)
            self.visit(a, guard if cg is None else g_and(guard, is_true(cg)))
            self.visit(b, guard if cg is None else g_and(guard, not_true(cg)))
        elif t == "call" and node["name"] == "COALESCE":
            rest = guard
            for arg in node["args"]:
                self.visit(arg, rest)
                leaf = self._value_leaf(arg)
                rest = rest if leaf is None else g_and(rest, is_null(leaf))
        else:
            for v in node.values():
                self.visit(v, guard)

    def _case(self, node, guard):
        rest = guard
        operand = node.get("operand")
        if operand is not None:
            self.visit(operand, guard)
        for cond, val in node["whens"]:
            test = cond if operand is None else {"type": "binary", "op": "=", "left": operand, "right": cond}
            self.visit(test, rest)
            cg = self.compile(test)
            if cg is None:
                self.visit(val, rest)
                continue
            self.visit(val, g_and(rest, is_true(cg)))
            rest = g_and(rest, not_true(cg))
        if node.get("else") is not None:
            self.visit(node["else"], rest)
