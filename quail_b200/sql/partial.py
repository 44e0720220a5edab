"""Conditions decided on an AI.MAP or AI.EXTRACT answer while the model is still writing it.

The text decoded so far, `w`, limits the complete answers still possible,
C(w): every text that starts with `w` (the answer may also end right here).
A WHERE test q of the answer alone is decided TRUE at `w` when q(z) is TRUE
for every z in C(w), and decided NOT TRUE when q(z) is FALSE or NULL for every
z; otherwise it is undecided. The region stops decoding an answer once its
test is decided NOT TRUE (the row is dropped whatever the rest of the answer
says), and, when nothing else in the query reads the answer, once it is
decided TRUE (the row is kept whatever the rest says). The answer then holds
its text so far, which is one of C(w), so evaluating the test on it gives the
decided value.

`decide` evaluates a condition over C(w) rather than one value: every part of
the expression gets an abstract value saying what is known of it for all of
C(w):

  Known   one value (literals, and functions of known values);
  Text    the answer, or LOWER / UPPER / LEFT / SUBSTR(.., 1, k) of it: a text
          that starts with a known prefix, possibly cut at k characters;
  Count   LENGTH of a Text: an integer between two bounds;
  Truth   which of TRUE, FALSE and NULL are possible (comparisons, LIKE /
          ILIKE, STARTS_WITH, IN, IS NULL, AND, OR, NOT);
  Unknown anything else (a function this module has no rule for).

Every rule over-approximates the possible values, so a test is only ever
decided when it really is; parts are combined one at a time, ignoring that
two parts read the same answer, which can only leave more undecided.

Reference: crates/quail-datafusion/src/derive/partial.rs (conditions decided
on partial answers: the same decision states, C(w), and the same function
list) and quail/execution/answer_stops.py (when an answer stops). The
abstract values and their rules here are this build's own.
"""

from __future__ import annotations

from dataclasses import dataclass

TRUE, NOT_TRUE, UNDECIDED = "true", "not_true", "undecided"
ALL = frozenset((True, False, None))


@dataclass(frozen=True)
class Completions:
    """C(w): the answer's text so far and how it may go on."""

    prefix: str
    complete: bool = False           # the answer is finished: C(w) is the text alone
    may_be_null: bool = False
    max_chars: int | None = None     # the most characters the answer may still add


@dataclass(frozen=True)
class Known:
    value: object


@dataclass(frozen=True)
class Text:
    c: Completions
    case: str | None = None          # "lower" / "upper" applied to the answer
    cut: int | None = None           # at most this many characters kept

    def head(self) -> str:
        """The prefix every non-NULL value starts with."""
        p = self.c.prefix
        if self.case == "lower":
            p = p.lower()
        elif self.case == "upper":
            p = p.upper()
        return p if self.cut is None else p[:self.cut]

    def exact(self) -> bool:
        """Whether every non-NULL value is the one text head()."""
        if self.c.complete or self.c.max_chars == 0:
            return True
        return self.cut is not None and len(self.head()) >= self.cut

    def can_be(self, v: str) -> bool:
        h = self.head()
        if self.exact():
            return v == h
        if not v.startswith(h) or (self.cut is not None and len(v) > self.cut):
            return False
        return self.c.max_chars is None or len(v) - len(h) <= self.c.max_chars


@dataclass(frozen=True)
class Count:
    lo: int
    hi: int | None                   # None: no upper bound
    null: bool = False


@dataclass(frozen=True)
class Truth:
    values: frozenset


UNKNOWN = Truth(ALL)          # an unknown value: as a truth, anything


def _after(text: str) -> str | None:
    """The least string above every string that starts with `text`."""
    chars = list(text)
    while chars:
        c = ord(chars.pop())
        if c < 0x10FFFF:
            return "".join(chars) + chr(c + 1)
    return None


def _not(v):
    return None if v is None else not v


def _and(a, b):
    if a is False or b is False:
        return False
    if a is None or b is None:
        return None
    return True


def _or(a, b):
    if a is True or b is True:
        return True
    if a is None or b is None:
        return None
    return False


def _truth(x) -> frozenset:
    if isinstance(x, Truth):
        return x.values
    if isinstance(x, Known):
        v = x.value
        return frozenset((None if v is None else bool(v),))
    return ALL


def _compare_known(op: str, a, b):
    if a is None or b is None:
        return None
    try:
        return {"=": a == b, "<>": a != b, "!=": a != b, "<": a < b, "<=": a <= b,
                ">": a > b, ">=": a >= b}[op]
    except TypeError:
        return None


_FLIP = {"<": ">", "<=": ">=", ">": "<", ">=": "<=", "=": "=", "<>": "<>", "!=": "!="}


def _compare_text(op: str, t: Text, v) -> frozenset:
    """Possible values of (answer-derived text) op v for a known v."""
    out = {None} if t.c.may_be_null else set()
    if v is None:
        return frozenset({None})
    if not isinstance(v, str):
        return ALL
    h, exact = t.head(), t.exact()
    if exact:
        out.add(_compare_known(op, h, v))
        return frozenset(out)
    up = _after(h)
    below = up is not None and up <= v        # every non-NULL value is < v
    if op in ("=", "<>", "!="):
        eq_possible = t.can_be(v)
        out |= {True, False} if eq_possible else {op != "="}
        return frozenset(out)
    if op == "<":
        if h < v:
            out.add(True)
        if not below:
            out.add(False)
    elif op == "<=":
        if h <= v:
            out.add(True)
        if not below:
            out.add(False)
    elif op == ">":
        if not below:
            out.add(True)
        if h <= v:
            out.add(False)
    elif op == ">=":
        if not below:
            out.add(True)
        if h < v:
            out.add(False)
    else:
        return ALL
    return frozenset(out)


def _compare_count(op: str, n: Count, v) -> frozenset:
    if v is None or not isinstance(v, (int, float)) or isinstance(v, bool):
        return ALL if v is not None else frozenset({None})
    out = {None} if n.null else set()
    lo, hi = n.lo, n.hi
    # the values are the integers in [lo, hi]: each op holds for some and fails for some
    tests = {
        "=": (lo <= v and (hi is None or v <= hi), not (hi is not None and lo == hi == v)),
        "<": (lo < v, hi is None or hi >= v),
        "<=": (lo <= v, hi is None or hi > v),
        ">": (hi is None or hi > v, lo <= v),
        ">=": (hi is None or hi >= v, lo < v),
    }
    if op in ("<>", "!="):
        t, f = tests["="]
        t, f = f, t
    elif op in tests:
        t, f = tests[op]
    else:
        return ALL
    if t:
        out.add(True)
    if f:
        out.add(False)
    return frozenset(out)


def _like_states(pattern: str, text: str, ci: bool):
    """Pattern positions reachable after matching all of `text` (LIKE: % any run, _ one
    character, backslash escapes), and the parsed pattern."""
    toks = []
    i = 0
    while i < len(pattern):
        ch = pattern[i]
        if ch == "\\" and i + 1 < len(pattern):
            toks.append(("lit", pattern[i + 1]))
            i += 2
            continue
        toks.append(("any",) if ch == "%" else ("one",) if ch == "_" else ("lit", ch))
        i += 1
    if ci:
        toks = [(k, *(x.lower() for x in rest)) for k, *rest in toks]
        text = text.lower()

    def close(states):
        out = set(states)
        stack = list(states)
        while stack:
            s = stack.pop()
            if s < len(toks) and toks[s][0] == "any" and s + 1 not in out:
                out.add(s + 1)
                stack.append(s + 1)
        return out
    states = close({0})
    for ch in text:
        nxt = set()
        for s in states:
            if s >= len(toks):
                continue
            k = toks[s]
            if k[0] == "any":
                nxt.add(s)
            elif k[0] == "one" or k[1] == ch:
                nxt.add(s + 1)
        states = close(nxt)
        if not states:
            break
    return states, toks


def _like(t: Text, pattern, ci: bool, negated: bool) -> frozenset:
    if pattern is None:
        return frozenset({None})
    if not isinstance(pattern, str):
        return ALL
    out = {None} if t.c.may_be_null else set()
    h = t.head()
    states, toks = _like_states(pattern, h, ci)
    if t.exact():
        out.add((len(toks) in states) != negated)
        return frozenset(out)
    if not states:
        out.add(negated)                  # no text starting with the prefix matches
    elif any(s < len(toks) and all(k[0] == "any" for k in toks[s:]) for s in states):
        out.add(not negated)              # every text starting with the prefix matches
    else:
        out |= {True, False}
    return frozenset(out)


def _starts_with(t: Text, s) -> frozenset:
    if s is None:
        return frozenset({None})
    if not isinstance(s, str):
        return ALL
    out = {None} if t.c.may_be_null else set()
    h = t.head()
    if h.startswith(s):
        out.add(True)
    elif t.exact() or not s.startswith(h):
        out.add(False)
    else:
        out |= {True, False}
    return frozenset(out)


class _Eval:
    def __init__(self, answer_key: str, c: Completions, key_of, field: str | None = None):
        self.key = answer_key
        self.c = c
        self.key_of = key_of
        self.field = field            # an extraction's struct field the answer is (None: the call itself)

    def __call__(self, e):
        t = e.get("type")
        if t == "literal":
            return Known(e.get("value"))
        if t == "call" and e.get("name") == "HINT":
            return self(e["args"][0])
        if (self.field is not None and t == "subscript" and isinstance(e.get("arg"), dict)
                and self.key_of(e["arg"]) == self.key):
            idx = e.get("index", {})
            return Text(self.c) if idx.get("type") == "literal" and idx.get("value") == self.field else UNKNOWN
        if t == "call" and self.key_of(e) == self.key:
            return Text(self.c) if self.field is None else UNKNOWN
        if t == "unary" and e.get("op") == "NOT":
            return Truth(frozenset(_not(v) for v in _truth(self(e["arg"]))))
        if t == "unary" and e.get("op") == "-":
            a = self(e["arg"])
            return Known(-a.value) if isinstance(a, Known) and isinstance(a.value, (int, float)) else UNKNOWN
        if t == "binary":
            return self._binary(e)
        if t == "like":
            a, p = self(e["arg"]), self(e["pattern"])
            ci, neg = bool(e.get("case_insensitive")), bool(e.get("negated"))
            if isinstance(a, Text) and isinstance(p, Known):
                return Truth(_like(a, p.value, ci, neg))
            return UNKNOWN
        if t == "in":
            if "query" in e:
                return UNKNOWN
            a = self(e["arg"])
            items = [self(x) for x in e.get("list", [])]
            if not all(isinstance(x, Known) for x in items):
                return UNKNOWN
            vals = [x.value for x in items]
            if not isinstance(a, Text):
                return UNKNOWN
            # IN is the OR of its equalities
            acc = {False}
            for v in vals:
                acc = {_or(x, y) for x in acc for y in _compare_text("=", a, v)}
            if e.get("negated"):
                acc = {_not(x) for x in acc}
            return Truth(frozenset(acc))
        if t == "is_null":
            a = self(e["arg"])
            neg = bool(e.get("negated"))
            if isinstance(a, Known):
                return Known((a.value is None) != neg)
            if isinstance(a, (Text, Count)):
                null = a.c.may_be_null if isinstance(a, Text) else a.null
                vals = {neg} | ({not neg} if null else set())
                return Truth(frozenset(vals))
            return UNKNOWN
        if t == "call":
            return self._call(e)
        return UNKNOWN

    def _binary(self, e):
        op = e.get("op")
        if op in ("AND", "OR"):
            a, b = _truth(self(e["left"])), _truth(self(e["right"]))
            f = _and if op == "AND" else _or
            return Truth(frozenset(f(x, y) for x in a for y in b))
        a, b = self(e["left"]), self(e["right"])
        if op not in _FLIP:
            if isinstance(a, Known) and isinstance(b, Known):
                try:
                    v = {"+": lambda: a.value + b.value, "-": lambda: a.value - b.value,
                         "*": lambda: a.value * b.value, "||": lambda: str(a.value) + str(b.value)}[op]()
                    return Known(v)
                except Exception:       # noqa: BLE001 - an operator this module has no rule for
                    return UNKNOWN
            return UNKNOWN
        if isinstance(a, Known) and not isinstance(b, Known):
            a, b, op = b, a, _FLIP[op]
        if isinstance(a, Known) and isinstance(b, Known):
            return Known(_compare_known(op, a.value, b.value))
        if not isinstance(b, Known):
            return UNKNOWN
        if isinstance(a, Text):
            return Truth(_compare_text(op, a, b.value))
        if isinstance(a, Count):
            return Truth(_compare_count(op, a, b.value))
        return UNKNOWN

    def _call(self, e):
        name = e.get("name", "").upper()
        args = [self(x) for x in e.get("args", [])]
        if all(isinstance(x, Known) for x in args):
            return self._known_call(name, [x.value for x in args])
        if name in ("LOWER", "UPPER") and len(args) == 1 and isinstance(args[0], Text):
            a = args[0]
            if a.case is None and a.cut is None:
                return Text(a.c, case=name.lower(), cut=None)
            return UNKNOWN
        if name in ("LEFT", "SUBSTR", "SUBSTRING") and args and isinstance(args[0], Text):
            a = args[0]
            if name == "LEFT" and len(args) == 2 and isinstance(args[1], Known):
                k = args[1].value
            elif (name != "LEFT" and len(args) == 3 and isinstance(args[1], Known) and args[1].value == 1
                  and isinstance(args[2], Known)):
                k = args[2].value
            else:
                return UNKNOWN
            if not isinstance(k, int) or k < 0:
                return UNKNOWN
            return Text(a.c, a.case, k if a.cut is None else min(a.cut, k))
        if name in ("LENGTH", "CHAR_LENGTH", "CHARACTER_LENGTH") and len(args) == 1 and isinstance(args[0], Text):
            a = args[0]
            h = a.head()
            if a.exact():
                return Count(len(h), len(h), a.c.may_be_null)
            hi = None if a.c.max_chars is None else len(h) + a.c.max_chars
            if a.cut is not None:
                hi = a.cut if hi is None else min(hi, a.cut)
            return Count(len(h), hi, a.c.may_be_null)
        if name == "STARTS_WITH" and len(args) == 2 and isinstance(args[0], Text) and isinstance(args[1], Known):
            return Truth(_starts_with(args[0], args[1].value))
        return UNKNOWN

    @staticmethod
    def _known_call(name: str, vals: list):
        try:
            if name == "LOWER":
                return Known(None if vals[0] is None else str(vals[0]).lower())
            if name == "UPPER":
                return Known(None if vals[0] is None else str(vals[0]).upper())
            if name in ("LENGTH", "CHAR_LENGTH", "CHARACTER_LENGTH"):
                return Known(None if vals[0] is None else len(str(vals[0])))
        except Exception:               # noqa: BLE001 - fall back to unknown
            pass
        return UNKNOWN


def decide(expr: dict, answer_key: str, completions: Completions, key_of, field: str | None = None) -> str:
    """TRUE, NOT_TRUE or UNDECIDED for condition `expr` over the answers C(w) of the model
    call whose key (`key_of(node)`) is `answer_key` (with `field`: of that extraction's field,
    read as `call['field']`)."""
    vals = _truth(_Eval(answer_key, completions, key_of, field)(expr))
    if vals == frozenset({True}):
        return TRUE
    if True not in vals:
        return NOT_TRUE
    return UNDECIDED


def reads_answer_alone(expr: dict, answer_key: str, key_of) -> bool:
    """Whether `expr` reads nothing of the row but the answer of call `answer_key` (no column,
    no other model call, no subquery): its decision then holds for every row alike."""
    def ok(n) -> bool:
        if isinstance(n, list):
            return all(ok(x) for x in n)
        if not isinstance(n, dict):
            return True
        t = n.get("type")
        if t == "call" and n.get("name") == "HINT":
            return ok(n["args"][0])
        if t == "call" and key_of(n) == answer_key:
            return True
        if t in ("column", "star", "scalar_subquery", "exists", "in_subquery", "subquery"):
            return False
        return all(ok(v) for k, v in n.items() if k != "type")
    return ok(expr)


def extraction_prefix(text: str) -> str | None:
    """The text every complete extraction answer starts with, given its decoded text so far
    (the answer is the text stripped, without a leading "Phrase:"), or None while that is not
    known yet (the text so far could still become the "Phrase:" label)."""
    s = partial_text(text).strip()
    low = s.lower()
    if len(s) < 7 and "phrase:".startswith(low):
        return None
    if low.startswith("phrase:"):
        s = s[7:].strip()
    return s


def extraction_field(expr: dict, answer_key: str, key_of) -> str | None:
    """The one struct field `expr` reads of the extraction `answer_key` (every read is
    call['field'] with the same literal field), or None."""
    fields = set()
    bare = [False]

    def visit(n, under_subscript=False):
        if isinstance(n, list):
            for x in n:
                visit(x)
            return
        if not isinstance(n, dict):
            return
        if n.get("type") == "subscript" and isinstance(n.get("arg"), dict) and key_of(n["arg"]) == answer_key:
            idx = n.get("index", {})
            if idx.get("type") == "literal" and isinstance(idx.get("value"), str):
                fields.add(idx["value"])
            else:
                bare[0] = True
            return
        if n.get("type") == "call" and key_of(n) == answer_key:
            bare[0] = True
            return
        for k, v in n.items():
            if k != "type":
                visit(v)
    visit(expr)
    return fields.pop() if len(fields) == 1 and not bare[0] else None


def partial_text(text: str) -> str:
    """The text of an answer's tokens so far up to its last whole character."""
    return text.rstrip("\ufffd")
