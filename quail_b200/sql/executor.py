"""Binding and running a parsed query over Arrow tables, with AI calls on the model.

The C++ parser (quail_b200._native.parse_sql) gives a JSON tree; this module
binds names against the session's tables and runs the relational operators
with pyarrow (scans, hash joins, filters, projections, aggregates, sorts,
limits). AI calls are the reference's logical rules in small
(crates/quail-datafusion/src/rules):

- lowering: each AI.* call in WHERE, SELECT, ORDER BY or HAVING becomes a
  model call bound to a prompt (`quail_b200.api.prompts`);
- placement / guards: WHERE conjuncts without AI calls run first, so the
  model sees only the rows they keep; AI.IF conjuncts then run as a guarded
  chain (each later call only on the rows every earlier filter kept); the
  SELECT / ORDER BY calls run on the survivors, next to them;
- merge: identical calls (same function, prompt and document column) are
  evaluated once per row, and identical documents once per table
  (`ModelEngine.run_region` deduplicates).

- demand (`quail_b200.sql.guards`): a call under a CASE branch, the right
  side of AND / OR, IFF or COALESCE is asked only on the rows whose guard
  holds (CASE guards and OR guards, crates/quail-datafusion/src/rules/
  guards.rs, or_guards.rs); all of one document's calls share a region,
  the guarded ones after the calls their guards read;
- fetch (rules/derive/fetch.rs): with LIMIT (and no ORDER BY, or one on
  plain columns, which is applied first) the rows go to the model in
  slices, and no further slice is asked once LIMIT rows came through;
- streaming (crates/quail/src/lib.rs:376 sql_stream): `Executor.stream`
  yields each slice's rows as its region finishes.

`SET quail.pushdown = false` turns demand and fetch off: every call is then
asked on every row that reaches its operator (the transcript tests compare
both ways: same rows, fewer questions with the rules on).
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass, field

import numpy as np
import pyarrow as pa
import pyarrow.compute as pc

from quail_b200.api import prompts as P

# AI.SAE_FEATURES' type: one {feature, strength} struct per nonzero feature, strongest first
FEATURE_LIST = pa.list_(pa.struct([("feature", pa.int32()), ("strength", pa.float32())]))

CPU_AI_FUNCTIONS = ("AI.PARSE_DOCUMENT", "AI.PDF_PAGES", "AI.IMAGE")
# Snowflake spellings of the document functions
CPU_ALIASES = {"AI_PARSE_DOCUMENT": "AI.PARSE_DOCUMENT", "AI_PDF_PAGES": "AI.PDF_PAGES", "AI_IMAGE": "AI.IMAGE"}
MODEL_AI_FUNCTIONS = ("AI.IF", "AI_FILTER", "AI.SCORE", "AI.CLASSIFY", "AI.EXTRACT", "AI.EXTRACT_SPAN",
                      "AI.MAP", "AI.SAE_FEATURES")
AGGREGATES = ("COUNT", "SUM", "AVG", "MIN", "MAX", "ARRAY_AGG", "ANY_VALUE")
MAP_MAX_TOKENS_LIMIT = 32_768
MAP_DEFAULT_TOKENS = 256


class QueryError(ValueError):
    pass


def parse(text: str) -> dict:
    from quail_b200 import _native
    return json.loads(_native.parse_sql(text))


# ---------------------------------------------------------------- expression helpers

def walk(node):
    """Yield every dict node of a tree."""
    if isinstance(node, dict):
        yield node
        for v in node.values():
            yield from walk(v)
    elif isinstance(node, list):
        for v in node:
            yield from walk(v)


def is_model_call(node) -> bool:
    return isinstance(node, dict) and node.get("type") == "call" and node.get("name") in MODEL_AI_FUNCTIONS


def has_model_call(node) -> bool:
    return any(is_model_call(n) for n in walk(node))


def is_aggregate(node) -> bool:
    return isinstance(node, dict) and node.get("type") == "call" and node.get("name") in AGGREGATES


def conjuncts(node) -> list:
    if node is None:
        return []
    if node.get("type") == "binary" and node.get("op") == "AND":
        return conjuncts(node["left"]) + conjuncts(node["right"])
    return [node]


def node_key(node) -> str:
    return json.dumps(node, sort_keys=True)


def expr_name(node) -> str:
    t = node.get("type")
    if t == "column":
        return node["name"]
    if t == "call":
        return node["name"].lower()
    if t == "literal":
        return str(node["value"])
    return t


def literal_value(node):
    if node is None:
        return None
    t = node.get("type")
    if t == "literal":
        return node["value"]
    if t == "array":
        return [literal_value(x) for x in node["items"]]
    if t == "object":
        return {k: literal_value(v) for k, v in node["items"]}
    if t == "unary" and node["op"] == "-":
        v = literal_value(node["arg"])
        return -v if isinstance(v, (int, float)) else None
    raise QueryError(f"expected a constant, got {t}")


# ---------------------------------------------------------------- relations

@dataclass
class Relation:
    """An Arrow table whose columns are addressed as (qualifier, name)."""

    table: pa.Table
    cols: list  # [(qualifier or None, name)] parallel to table columns

    @classmethod
    def from_table(cls, t: pa.Table, qualifier: str | None) -> "Relation":
        names = t.column_names
        return cls(t.rename_columns([f"c{i}" for i in range(len(names))]), [(qualifier, n) for n in names])

    @property
    def num_rows(self) -> int:
        return self.table.num_rows

    def resolve(self, qualifier: str | None, name: str) -> int:
        hits = [i for i, (q, n) in enumerate(self.cols)
                if n.lower() == name.lower() and (qualifier is None or (q or "").lower() == qualifier.lower())]
        if not hits:
            raise QueryError(f"unknown column {qualifier + '.' if qualifier else ''}{name}")
        if len(hits) > 1:
            exact = [i for i in hits if self.cols[i][1] == name]
            if len(exact) == 1:
                return exact[0]
            raise QueryError(f"ambiguous column {name}")
        return hits[0]

    def column(self, i: int):
        return self.table.column(i)

    def take(self, idx) -> "Relation":
        return Relation(self.table.take(idx), list(self.cols))

    def filter(self, mask) -> "Relation":
        return Relation(self.table.filter(mask), list(self.cols))

    def with_column(self, arr, qualifier, name) -> "Relation":
        t = self.table.append_column(f"c{len(self.cols)}", arr)
        return Relation(t, self.cols + [(qualifier, name)])


def concat_relations(left: Relation, right: Relation) -> Relation:
    t = left.table
    for i in range(right.table.num_columns):
        t = t.append_column(f"c{t.num_columns}", right.table.column(i))
    return Relation(t.rename_columns([f"c{i}" for i in range(t.num_columns)]), left.cols + right.cols)


# ---------------------------------------------------------------- AI call binding

@dataclass
class BoundCall:
    """An AI call ready for the engine: which rows' documents, which prompt."""

    key: str
    kind: str                   # filter | score | classify | map | extract
    preamble: str
    tail: str
    doc_expr: dict              # expression giving each row's document
    labels: list = field(default_factory=list)
    max_tokens: int = MAP_DEFAULT_TOKENS
    probabilities: bool = False
    selectivity: float | None = None
    questions: list = field(default_factory=list)   # extract: one call per question
    fields: list | None = None                       # extract: struct field names ({'name': question} form)
    span: bool = False
    pooling: str = "last"                            # features
    descriptions: list = field(default_factory=list)  # classify: per-label descriptions
    segments: list | None = None                     # decision prompts: the tail's segments
    read: list = field(default_factory=list)         # decision prompts: segments the head reads
    letters: list = field(default_factory=list)      # lettered prompts: option i's answer letter
    drops: bool = True                               # filter: FALSE drops the row (WHERE chains)
    guard: dict | None = None                        # demand guard (quail_b200.sql.guards)
    stop: dict | None = None                         # map: WHERE test decided on partial answers


def _options(node) -> dict:
    if node is None:
        return {}
    v = literal_value(node)
    if not isinstance(v, dict):
        raise QueryError("AI function options must be an object such as {'selectivity': 0.3}")
    return v


def _prompt_parts(arg) -> tuple[str, dict, int]:
    """(template, document expression, number of documents) of a PROMPT(...) or a plain column."""
    if arg.get("type") == "call" and arg["name"] == "PROMPT":
        args = arg["args"]
        if not args or args[0].get("type") != "literal" or args[0]["kind"] != "string":
            raise QueryError("PROMPT takes a template string first")
        template = args[0]["value"]
        values = args[1:]
        P.check_placeholders(template, len(values))
        if len(values) == 1:
            return template, values[0], 1
        if len(values) == 0:
            return template, {"type": "literal", "kind": "string", "value": ""}, 0
        # several values: one computed document, DOCUMENT k labels in order
        parts = []
        for i, v in enumerate(values):
            label = {"type": "literal", "kind": "string", "value": f"DOCUMENT {i + 1}:\n" if i == 0 else
                     f"\n\nDOCUMENT {i + 1}:\n"}
            parts += [label, v]
        doc = parts[0]
        for p in parts[1:]:
            doc = {"type": "binary", "op": "||", "left": doc, "right": p}
        tmpl = re.sub(r"\{\d+\}", "", template).strip()
        return tmpl + " {0}", doc, len(values)
    return "{0}", arg, 1


def _refuse(reason: str, constraint: str):
    from quail_b200.api.config import Refusal, RefusalError
    raise RefusalError(Refusal(reasons=(reason,), constraint=constraint))


def bind_role_call(node, model: P.PromptModel) -> BoundCall:
    """A call on a reranker or a decision model: their own prompts, their own readouts.

    Reranker: AI.SCORE only (crates/quail-planner/src/graph.rs:1719-1738).
    Decision: AI.IF / AI_FILTER / AI.SCORE read the No and Yes options,
    AI.CLASSIFY one option per label; neither decodes text
    (validation.rs:207-231).
    """
    name = node["name"]
    args = [a for a in node["args"] if a.get("type") != "named_arg"]
    named = {a["name"].lower(): a["value"] for a in node["args"] if a.get("type") == "named_arg"}
    key = node_key(node)
    if name in ("AI.MAP", "AI.EXTRACT", "AI.EXTRACT_SPAN"):
        _refuse(f"{name} decodes the model's next tokens, which {model.name!r} does not give",
                f"unsupported_{name[3:].lower()}_query")
    if model.role == "reranker":
        if name == "AI.CLASSIFY":
            _refuse("a reranker model cannot run AI.CLASSIFY", "reranker_only_scores")
        if name != "AI.SCORE":
            _refuse("a reranker model can only be used with AI.SCORE", "reranker_only_scores")
        if not args:
            raise QueryError(f"{name} takes a prompt")
        template, doc, ndocs = _prompt_parts(args[0])
        if ndocs > 1:
            raise QueryError("AI.SCORE on a reranker reads one document")
        bp = P.bind_reranker_prompt(template)
        return BoundCall(key=key, kind="score", preamble=bp.preamble, tail=bp.tail, doc_expr=doc)
    lettered = model.layout == "mammoth"
    if name in ("AI.IF", "AI_FILTER", "AI.SCORE"):
        if not args:
            raise QueryError(f"{name} takes a prompt")
        template, doc, _ = _prompt_parts(args[0])
        opts = _options(args[1] if len(args) > 1 else named.get("options"))
        kind = "score" if name == "AI.SCORE" else "filter"
        if lettered:
            bp = P.bind_mammoth_prompt(template, kind, model.turn)
            return BoundCall(key=key, kind=kind, preamble=bp.preamble, tail=bp.tail, doc_expr=doc,
                             selectivity=opts.get("selectivity"), letters=bp.letters)
        bp = P.bind_decision_prompt(template, kind, model.turn)
        return BoundCall(key=key, kind=kind, preamble=bp.preamble, tail=bp.tail, doc_expr=doc,
                         selectivity=opts.get("selectivity"), segments=bp.segments, read=bp.read)
    if name == "AI.CLASSIFY":
        call = bind_call(node, model.turn)
        opts = _options(args[2] if len(args) > 2 else named.get("options"))
        template, _, _ = _prompt_parts(args[0])
        if lettered:
            try:
                bp = P.bind_mammoth_choice_prompt(template if template != "{0}" else None, call.labels,
                                                  call.descriptions, opts.get("task_description", ""), model.turn)
            except P.PromptError as exc:
                raise QueryError(str(exc)) from None
            call.preamble, call.tail, call.letters = bp.preamble, bp.tail, bp.letters
            return call
        bp = P.bind_decision_choice_prompt(template if template != "{0}" else None, call.labels,
                                           call.descriptions, opts.get("task_description", ""), model.turn)
        call.preamble, call.tail, call.segments, call.read = bp.preamble, bp.tail, bp.segments, bp.read
        return call
    return bind_call(node, model.turn)


def bind_set_call(node, model: P.PromptModel) -> BoundCall:
    """An AI call for a set-attention model (the d1 layout): yes / no questions, option codes
    and pointer reads, asked in passes over each document; nothing decodes text
    (crates/quail-planner/src/prompts.rs:174-189, 940-990)."""
    name = node["name"]
    args = [a for a in node["args"] if a.get("type") != "named_arg"]
    named = {a["name"].lower(): a["value"] for a in node["args"] if a.get("type") == "named_arg"}
    key = node_key(node)
    if name in ("AI.MAP", "AI.SAE_FEATURES"):
        _refuse(f"{name} needs text decoding or features, which the set-attention model {model.name!r} does not "
                f"give", f"unsupported_{name[3:].lower()}_query")
    if name in ("AI.IF", "AI_FILTER", "AI.SCORE"):
        if not args:
            raise QueryError(f"{name} takes a prompt")
        template, doc, _ = _prompt_parts(args[0])
        opts = _options(args[1] if len(args) > 1 else named.get("options"))
        kind = "score" if name == "AI.SCORE" else "filter"
        bp = P.bind_d1_prompt(template, kind, model.turn)
        return BoundCall(key=key, kind=kind, preamble=bp.preamble, tail=bp.tail, doc_expr=doc,
                         selectivity=opts.get("selectivity"))
    if name == "AI.CLASSIFY":
        call = bind_call(node, model.turn)
        opts = _options(args[2] if len(args) > 2 else named.get("options"))
        template, _, _ = _prompt_parts(args[0])
        bp = P.bind_d1_choice_prompt(template if template != "{0}" else None, call.labels, call.descriptions,
                                     opts.get("task_description", ""), model.turn)
        call.preamble, call.tail, call.letters = bp.preamble, bp.tail, bp.letters
        return call
    if name in ("AI.EXTRACT", "AI.EXTRACT_SPAN"):
        call = bind_call(node, model.turn)
        try:
            bp = P.bind_d1_read_prompt(call.questions[0], model.turn)
        except P.PromptError as exc:
            raise QueryError(str(exc)) from None
        call.preamble, call.tail = bp.preamble, bp.tail
        return call
    return bind_call(node, model.turn)


def bind_call(node, turn: P.Turn, model: P.PromptModel | None = None) -> BoundCall:
    if model is not None and model.layout == "d1":
        return bind_set_call(node, model)
    if model is not None and model.role in ("reranker", "decision"):
        return bind_role_call(node, model)
    name = node["name"]
    args = [a for a in node["args"] if a.get("type") != "named_arg"]
    named = {a["name"].lower(): a["value"] for a in node["args"] if a.get("type") == "named_arg"}
    key = node_key(node)
    if name in ("AI.IF", "AI_FILTER", "AI.SCORE"):
        if not args:
            raise QueryError(f"{name} takes a prompt")
        template, doc, ndocs = _prompt_parts(args[0])
        opts = _options(args[1] if len(args) > 1 else named.get("options"))
        bp = P.bind_prompt(template if ndocs <= 1 else template, 1, turn)
        kind = "score" if name == "AI.SCORE" else "filter"
        return BoundCall(key=key, kind=kind, preamble=bp.preamble, tail=bp.tail, doc_expr=doc,
                         selectivity=opts.get("selectivity"))
    if name == "AI.CLASSIFY":
        if len(args) < 2:
            raise QueryError("AI.CLASSIFY takes an input and a list of categories")
        template, doc, _ = _prompt_parts(args[0])
        cats = literal_value(args[1])
        if not isinstance(cats, list) or not cats:
            raise QueryError("AI.CLASSIFY categories must be a non-empty array literal")
        labels, descriptions = [], []
        for c in cats:
            if isinstance(c, dict):
                labels.append(str(c.get("label")))
                descriptions.append(str(c.get("description", "")))
            else:
                labels.append(str(c))
                descriptions.append("")
        if len(set(labels)) != len(labels):
            raise QueryError("AI.CLASSIFY categories must be distinct")
        opts = _options(args[2] if len(args) > 2 else named.get("options"))
        if model is not None and model.layout == "letters":
            # a canvas model reads one row: the labels are listed under letters, answered by a letter
            try:
                bp = P.bind_letters_classify_prompt(template if template != "{0}" else None, labels, descriptions,
                                                    opts.get("task_description", ""), turn)
            except P.PromptError as exc:
                raise QueryError(str(exc)) from None
            return BoundCall(key=key, kind="classify", preamble=bp.preamble, tail=bp.tail, doc_expr=doc,
                             labels=labels, probabilities=bool(opts.get("probabilities", False)),
                             descriptions=descriptions, letters=bp.letters)
        bp = P.bind_classify_prompt(template if template != "{0}" else None, labels, descriptions,
                                    opts.get("task_description", ""), turn)
        return BoundCall(key=key, kind="classify", preamble=bp.preamble, tail=bp.tail, doc_expr=doc, labels=labels,
                         probabilities=bool(opts.get("probabilities", False)), descriptions=descriptions)
    if name == "AI.MAP":
        if len(args) < 2:
            raise QueryError("AI.MAP takes an input and an instruction")
        _, doc, _ = _prompt_parts(args[0])
        instruction = literal_value(args[1])
        max_tokens = literal_value(args[2]) if len(args) > 2 else MAP_DEFAULT_TOKENS
        if not isinstance(max_tokens, int) or not 1 <= max_tokens <= MAP_MAX_TOKENS_LIMIT:
            raise QueryError(f"AI.MAP max_tokens must be an integer in [1, {MAP_MAX_TOKENS_LIMIT}]")
        bp = P.bind_map_prompt(str(instruction), turn)
        return BoundCall(key=key, kind="map", preamble=bp.preamble, tail=bp.tail, doc_expr=doc, max_tokens=max_tokens)
    if name in ("AI.EXTRACT", "AI.EXTRACT_SPAN"):
        if len(args) < 2:
            raise QueryError(f"{name} takes an input and a list of questions")
        _, doc, _ = _prompt_parts(args[0])
        qs = literal_value(args[1])
        fields = None
        if isinstance(qs, dict):
            # {'field': 'question', ...}: a struct with one field per question
            if not qs or not all(isinstance(k, str) and k for k in qs):
                raise QueryError(f"{name} questions must map field names to questions")
            fields, qs = list(qs), [str(v) for v in qs.values()]
        elif isinstance(qs, str):
            qs = [qs]
        elif isinstance(qs, list) and qs:
            qs = [str(q) for q in qs]
        else:
            raise QueryError(f"{name} takes an object from field names to questions")
        bp = P.bind_extract_prompt(qs[0], turn)
        return BoundCall(key=key, kind="extract", preamble=bp.preamble, tail=bp.tail, doc_expr=doc, questions=qs,
                         fields=fields, span=name == "AI.EXTRACT_SPAN", max_tokens=64)
    if name == "AI.SAE_FEATURES":
        opts = _options(args[1]) if len(args) == 2 else {}
        pooling = opts.get("pooling")
        if len(args) != 2 or pooling not in ("last", "max"):
            raise QueryError("AI.SAE_FEATURES needs a PROMPT and pooling set to 'last' or 'max'.")
        template, doc, _ = _prompt_parts(args[0])
        try:
            bp = P.bind_features_prompt(template, turn)
        except P.PromptError as exc:
            raise QueryError(str(exc)) from None
        return BoundCall(key=key, kind="features", preamble=bp.preamble, tail=bp.tail, doc_expr=doc,
                         pooling=pooling)
    raise QueryError(f"unknown AI function {name}")


# ---------------------------------------------------------------- the executor

class Executor:
    def __init__(self, catalog: dict, engine=None, turn: P.Turn | None = None, settings: dict | None = None,
                 model: P.PromptModel | None = None):
        self.catalog = catalog
        self.engine = engine
        cfg = getattr(engine, "cfg", None)
        if model is None:
            model = P.prompt_model(cfg) if cfg is not None else P.PromptModel()
        if turn is not None:
            model = P.PromptModel(role=model.role, layout=model.layout, turn=turn, name=model.name)
        self.model = model
        self.turn = model.turn
        self.settings = settings or {}
        self.ctes: dict = {}
        self.report = {"regions": [], "asked": 0, "fresh_tokens": 0, "passes": 0, "evaluated_documents": 0}
        self.ai_values: dict = {}   # (call key) -> Arrow array aligned with the relation being evaluated
        self.carried = ({}, {})     # WHERE answers and their asked rows, aligned with the rows it kept
        self.asked_rows: dict = {}  # (call key) -> bool array: rows of ai_values[key] the call was asked on
        flag = self.settings.get("quail.pushdown", self.settings.get("pushdown", True))
        self.pushdown = str(flag).lower() not in ("false", "off", "0", "no")

    # ------------------------------------------------------------ entry
    def run(self, tree: dict) -> pa.Table:
        t = tree.get("type")
        if t == "explain":
            raise QueryError("EXPLAIN is answered by Query.explain()")
        self.check_similar(tree)
        # how often each model call is written in the whole statement (answer stops read it)
        self.call_counts: dict = {}
        for n in walk(tree):
            if is_model_call(n):
                self.call_counts[node_key(n)] = self.call_counts.get(node_key(n), 0) + 1
        return self.query(tree)

    def check_similar(self, tree: dict) -> None:
        """Refuse calls written the same but for case, whitespace or punctuation; warn of calls a
        typo apart (sql/similar.py)."""
        from quail_b200.sql import similar
        calls = [n for n in walk(tree) if is_model_call(n)]
        for kind, a, b in similar.similar_calls(calls):
            if kind == "spelling":
                raise QueryError(similar.message(kind, a, b))
            self.report.setdefault("warnings", []).append(similar.message(kind, a, b))
            from quail_b200.utils import progress
            progress.say(similar.message(kind, a, b))

    def query(self, node) -> pa.Table:
        saved = dict(self.ctes)
        for w in node.get("with", []):
            self.ctes[w["name"].lower()] = self.query(w["query"])
        if node["type"] == "union":
            left = self.query(node["left"])
            right = self.query(node["right"])
            right = right.rename_columns(left.column_names).cast(left.schema)
            out = pa.concat_tables([left, right])
            if not node["all"]:
                out = _distinct(out)
            out = self._order_limit_output(out, node)
        else:
            out = self.select(node)
        self.ctes = saved
        return out

    # ------------------------------------------------------------ FROM
    def table_ref(self, ref) -> Relation:
        alias = ref.get("alias")
        if ref["type"] == "subquery":
            return Relation.from_table(self.query(ref["query"]), alias)
        name = ref["name"]
        low = name.lower()
        if low in self.ctes:
            return Relation.from_table(self.ctes[low], alias or name)
        for k, prov in self.catalog.items():
            if k.lower() == low:
                t = prov.scan().read_all()
                return Relation.from_table(t, alias or name)
        raise QueryError(f"unknown table {name}; registered: {sorted(self.catalog)}")

    def from_clause(self, node) -> Relation:
        if "from" not in node:
            return Relation(pa.table({"c0": [0]}), [(None, "__dual")])
        rel = self.table_ref(node["from"][0])
        for j in node.get("joins", []):
            right = self.table_ref(j["table"])
            rel = self.join(rel, right, j)
        return rel

    def join(self, left: Relation, right: Relation, j) -> Relation:
        kind = j["kind"]
        on = j.get("on")
        if "using" in j:
            on = None
            for c in j["using"]:
                eq = {"type": "binary", "op": "=", "left": {"type": "column", "table": left.cols[left.resolve(None, c)][0],
                                                              "name": c},
                      "right": {"type": "column", "table": right.cols[right.resolve(None, c)][0], "name": c}}
                on = eq if on is None else {"type": "binary", "op": "AND", "left": on, "right": eq}
        if kind == "cross" or on is None:
            return self._cross(left, right)
        # equi-join keys between the two sides; the rest filters the joined rows
        keys, rest = [], []
        for c in conjuncts(on):
            pair = self._equi_pair(c, left, right)
            if pair is not None and not has_model_call(c):
                keys.append(pair)
            else:
                rest.append(c)
        if keys:
            lk = [f"c{i}" for i, _ in keys]
            rk = [f"c{i}" for _, i in keys]
            lt = left.table.append_column("__lrow", pa.array(np.arange(left.num_rows)))
            rt = right.table.append_column("__rrow", pa.array(np.arange(right.num_rows)))
            rt = rt.rename_columns([f"r{n}" for n in rt.column_names])
            jt = {"inner": "inner", "left": "left outer", "right": "right outer", "full": "full outer"}[kind]
            joined = lt.join(rt, keys=lk, right_keys=[f"r{k}" for k in rk], join_type=jt, coalesce_keys=False)
            li = joined.column("__lrow")
            ri = joined.column("r__rrow")
            lrel = Relation(left.table.take(li), list(left.cols))
            rrel = Relation(right.table.take(ri), list(right.cols))
            rel = concat_relations(lrel, rrel)
        else:
            if kind != "inner":
                raise QueryError(f"{kind.upper()} JOIN needs an equality condition")
            rel = self._cross(left, right)
        if rest and kind != "inner":
            raise QueryError("an outer join's ON may only hold equalities")
        # plain conditions first, then the model's: an AI condition over one column of each
        # side runs as pairs that share the anchor side's document KV
        for c in [c for c in rest if not has_model_call(c)] + [c for c in rest if has_model_call(c)]:
            pair = self._pair_call(c, left, right) if has_model_call(c) else None
            if pair is not None:
                rel = self._pair_filter(rel, *pair)
            else:
                rel = self.apply_where(rel, c)
        return rel

    # ------------------------------------------------------------ AI join on pairs
    def _side(self, e, left: Relation, right: Relation) -> str | None:
        """'L' or 'R' when every column of `e` belongs to that side only, else None."""
        sides = set()
        for n in walk(e):
            if n.get("type") == "column":
                in_l = in_r = True
                try:
                    left.resolve(n.get("table"), n["name"])
                except QueryError:
                    in_l = False
                try:
                    right.resolve(n.get("table"), n["name"])
                except QueryError:
                    in_r = False
                if in_l == in_r:
                    return None
                sides.add("L" if in_l else "R")
        return sides.pop() if len(sides) == 1 else None

    def _pair_call(self, c, left: Relation, right: Relation):
        """(call node, template, left expr, right expr, left placeholder) of an AI.IF over one
        document of each side, or None."""
        inner = c["args"][0] if c.get("type") == "call" and c["name"] == "HINT" else c
        if not (is_model_call(inner) and inner["name"] in ("AI.IF", "AI_FILTER")):
            return None
        if self.model.role in ("reranker", "decision"):
            return None
        args = [a for a in inner["args"] if a.get("type") != "named_arg"]
        if not args or args[0].get("type") != "call" or args[0]["name"] != "PROMPT":
            return None
        pargs = args[0]["args"]
        if len(pargs) != 3 or pargs[0].get("type") != "literal":
            return None
        s0, s1 = self._side(pargs[1], left, right), self._side(pargs[2], left, right)
        if {s0, s1} != {"L", "R"}:
            return None
        lexpr, rexpr = (pargs[1], pargs[2]) if s0 == "L" else (pargs[2], pargs[1])
        return inner, pargs[0]["value"], lexpr, rexpr, 0 if s0 == "L" else 1

    def _pair_filter(self, rel: Relation, node, template: str, lexpr, rexpr, lpos: int) -> Relation:
        """Keep the joined rows whose pair the model answers TRUE, asking each distinct pair once.

        The anchor side (the one whose documents are prefilled once and read by
        all of their pairs) is the one that makes the pair questions cheaper
        (`planner.search.choose_anchor`); with demand rules off every pair gets
        its own copy of its anchor document (the same prompt tokens, no sharing).
        """
        from quail_b200.planner.search import choose_anchor
        if rel.num_rows == 0:
            return rel
        ldocs = [None if v is None else str(v) for v in _as_array(self.eval(lexpr, rel), rel.num_rows).to_pylist()]
        rdocs = [None if v is None else str(v) for v in _as_array(self.eval(rexpr, rel), rel.num_rows).to_pylist()]
        P.check_placeholders(template, 2)
        question = re.sub(r"\{(\d+)\}", lambda m: f"DOCUMENT {int(m.group(1)) + 1}", template).strip()
        opts = _options(node["args"][1]) if len([a for a in node["args"] if a.get("type") != "named_arg"]) > 1 \
            else {}
        side = choose_anchor(ldocs, rdocs, opts.get("anchor"))
        self.report.setdefault("joins", []).append({"anchor": "left" if side == "L" else "right"})
        anc_docs, oth_docs = (ldocs, rdocs) if side == "L" else (rdocs, ldocs)
        anc_pos = lpos if side == "L" else 1 - lpos
        anc_label, oth_label = f"DOCUMENT {anc_pos + 1}:\n", f"\n\nDOCUMENT {2 - anc_pos}:\n"
        tail = P.JOIN_QUESTION_SEP + P.TASK_INSTRUCTION + question + P.ANSWER_CUE + self.turn.suffix
        anchors, where, pairs, pair_of = [], {}, [], {}
        keys = []
        for r in range(rel.num_rows):
            a = anc_label + (anc_docs[r] or "")
            o = oth_label + (oth_docs[r] or "")
            if self.pushdown:
                k = (a, o)
                if k in pair_of:            # a repeated pair is asked once
                    keys.append(pair_of[k])
                    continue
                if a not in where:
                    where[a] = len(anchors)
                    anchors.append(a)
                ai = where[a]
            else:
                ai = len(anchors)
                anchors.append(a)
                k = (ai, o)
            pair_of[k] = len(pairs)
            keys.append(len(pairs))
            pairs.append((ai, o))
        from quail_b200.api.engine import CallSpec
        spec = CallSpec(kind="filter", tail=tail, name=node_key(node))
        if self.engine is None:
            raise QueryError("this query needs a model; the session has none")
        out = self.engine.run_pairs(self.turn.prefix, anchors, pairs, spec)
        self._record(out.stats, "quail.ai_join")
        keep = [bool(out.values[keys[r]].get(spec.name)) for r in range(rel.num_rows)]
        return rel.filter(pa.array(keep))

    def _cross(self, left: Relation, right: Relation) -> Relation:
        n, m = left.num_rows, right.num_rows
        li = pa.array(np.repeat(np.arange(n), m))
        ri = pa.array(np.tile(np.arange(m), n))
        return concat_relations(Relation(left.table.take(li), list(left.cols)),
                                Relation(right.table.take(ri), list(right.cols)))

    def _equi_pair(self, c, left: Relation, right: Relation):
        if c.get("type") != "binary" or c.get("op") != "=":
            return None
        a, b = c["left"], c["right"]
        if a.get("type") != "column" or b.get("type") != "column":
            return None
        for x, y in ((a, b), (b, a)):
            try:
                i = left.resolve(x.get("table"), x["name"])
                k = right.resolve(y.get("table"), y["name"])
                return i, k
            except QueryError:
                continue
        return None

    # ------------------------------------------------------------ WHERE with AI placement
    def apply_where(self, rel: Relation, where) -> Relation:
        plain = [c for c in conjuncts(where) if not has_model_call(c)]
        ai = [c for c in conjuncts(where) if has_model_call(c)]
        for c in plain:
            rel = rel.filter(_as_mask(self.eval(c, rel)))
        return self.apply_ai_conjuncts(rel, ai)

    def apply_ai_conjuncts(self, rel: Relation, ai: list) -> Relation:
        """WHERE conjuncts holding model calls, on the rows the plain conjuncts kept."""
        if not ai:
            return rel
        # AI.IF conjuncts: a guarded chain; others evaluated on the survivors
        filters = []
        others = []
        for c in ai:
            inner = c
            if inner.get("type") == "call" and inner["name"] == "HINT":
                inner = inner["args"][0]
            if is_model_call(inner) and inner["name"] in ("AI.IF", "AI_FILTER"):
                filters.append(inner)
            else:
                others.append(c)
        if filters:
            from quail_b200.planner.search import doc_tokens, order_filters
            bound = [bind_call(f, self.turn, self.model) for f in filters]
            # cheapest-per-row-removed first: question tokens / (1 - hinted selectivity)
            order = order_filters([doc_tokens(b.tail) for b in bound],
                                  [b.selectivity if b.selectivity is not None else 0.5 for b in bound])
            rel = self.run_filters(rel, [bound[i] for i in order])
        carry: dict = {}
        carry_asked: dict = {}
        for c in others:
            pre = self._substring_precheck(rel, c)
            if pre is not None:
                rel = rel.filter(pre)
                keep = np.asarray(pre.to_pylist(), dtype=bool)
                carry = {k: v.filter(pre) for k, v in carry.items()}
                carry_asked = {k: a[keep] for k, a in carry_asked.items()}
            self.ai_values, self.asked_rows = dict(carry), dict(carry_asked)
            self.compute_ai(rel, [c], stops=self._answer_stops(c))
            mask = _as_mask(self.eval(c, rel))
            rel = rel.filter(mask)
            # the answers stay with the rows they belong to, with the rows each call was asked
            # on, so a later conjunct or the SELECT list reading the same call asks it only
            # where it was not asked yet
            keep = np.asarray(mask.to_pylist() if hasattr(mask, "to_pylist") else mask, dtype=bool)
            carry = {k: v.filter(mask) for k, v in self.ai_values.items()}
            carry_asked = {k: a[keep] for k, a in self.asked_rows.items() if k in carry}
            self.ai_values, self.asked_rows = {}, {}
        self.carried = (carry, carry_asked)
        return rel

    def _substring_precheck(self, rel: Relation, conjunct):
        """Rows whose document can give an extraction answer passing `conjunct`, or None.

        AI.EXTRACT copies each answer from its document, so an answer that must match a LIKE
        pattern needs a document containing the pattern's literal text: the longest run between
        wildcards, then that run's longest word (case and whitespace are where a decoded answer
        may differ from its document). `answer['f'] LIKE '%2027%'` then asks the model only on
        documents that contain '2027' (case-insensitively); the test itself still runs.
        Reference: crates/quail-datafusion/src/rules/substring.rs.
        """
        if not self.pushdown or rel.num_rows == 0 or conjunct.get("type") != "like" or conjunct.get("negated"):
            return None
        arg = conjunct["arg"]
        if arg.get("type") == "subscript":
            arg = arg["arg"]
        if not (is_model_call(arg) and arg["name"] == "AI.EXTRACT"):
            return None
        try:
            pat = literal_value(conjunct["pattern"])
        except QueryError:
            return None
        if not isinstance(pat, str):
            return None
        runs, cur, i = [], "", 0
        while i < len(pat):
            ch = pat[i]
            if ch == "\\" and i + 1 < len(pat):
                cur += pat[i + 1]
                i += 2
                continue
            if ch in "%_":
                runs.append(cur)
                cur = ""
            else:
                cur += ch
            i += 1
        runs.append(cur)
        words = max(runs, key=len).split()
        need = max(words, key=len) if words else ""
        if not need:
            return None
        b = bind_call(arg, self.turn, self.model)
        docs = _as_array(self.eval(b.doc_expr, rel), rel.num_rows)
        if not pa.types.is_string(docs.type) and not pa.types.is_large_string(docs.type):
            return None
        return pc.fill_null(pc.match_substring(docs, need, ignore_case=True), False)

    def _answer_stops(self, conjunct) -> dict:
        """The early stop of an AI.MAP answer that `conjunct` tests alone (quail_b200.sql.partial):
        {call key: {"test": conjunct, "when_true": nothing else reads the answer}}."""
        from quail_b200.sql import partial
        if not self.pushdown:
            return {}
        calls = {node_key(n): n for n in walk(conjunct) if is_model_call(n)}
        if len(calls) != 1:
            return {}
        (key, call), = calls.items()
        if call["name"] not in ("AI.MAP", "AI.EXTRACT") or not partial.reads_answer_alone(conjunct, key, node_key):
            return {}
        field = None
        if call["name"] == "AI.EXTRACT":
            # an extraction's test reads one field of its struct; that question's decode stops
            field = partial.extraction_field(conjunct, key, node_key)
            if field is None:
                return {}
        here = sum(1 for n in walk(conjunct) if is_model_call(n) and node_key(n) == key)
        total = getattr(self, "call_counts", {}).get(key)
        return {key: {"test": conjunct, "field": field, "when_true": total is not None and total == here}}

    def run_filters(self, rel: Relation, calls: list[BoundCall]) -> Relation:
        """AI.IF calls as one guarded chain over the relation's documents."""
        if rel.num_rows == 0 or not calls:
            return rel
        groups = {}
        for c in calls:
            groups.setdefault((c.preamble, node_key(c.doc_expr)), []).append(c)
        keep = np.ones(rel.num_rows, dtype=bool)
        for (_, _), cs in groups.items():
            docs = _documents(self.eval(cs[0].doc_expr, rel), rel.num_rows)
            idx = np.nonzero(keep)[0]
            vals = self._engine_region(cs[0].preamble, [docs[i] for i in idx], cs)
            for j, i in enumerate(idx):
                for c in cs:
                    if not vals[j].get(c.key, False):
                        keep[i] = False
        return rel.filter(pa.array(keep))

    def compute_ai(self, rel: Relation, exprs: list, stops: dict | None = None) -> None:
        """Evaluate the model calls inside `exprs` on `rel`, each on the rows its guard asks for.

        Calls reading the same document under the same instruction share a
        region. A guarded call comes after the calls its guard reads: in the
        same region (the guard is tested per row between the questions) or,
        for a call of another region, once that region's answers are in.
        """
        from quail_b200.sql import guards as G
        demand = G.Demand(self, rel, enabled=self.pushdown)
        for e in exprs:
            demand.visit(e)
        for k, (node, guard) in demand.guards.items():
            if k in self.ai_values:
                self._fill_unasked(rel, k, node, guard)
        todo = {k: v for k, v in demand.guards.items() if k not in self.ai_values}
        if not todo:
            return
        bound = {}
        for k, (node, guard) in todo.items():
            b = bind_call(node, self.turn, self.model)
            b.drops = False
            b.guard = None if guard["op"] == "true" else guard
            b.stop = (stops or {}).get(k)
            bound[k] = b
        n = rel.num_rows
        remaining = list(bound)
        while remaining:
            groups: dict = {}
            for k in remaining:
                b = bound[k]
                groups.setdefault((b.preamble, node_key(b.doc_expr)), []).append(k)
            ran = False
            for keys in groups.values():
                deps = set().union(*(G.calls_of(bound[k].guard) for k in keys))
                if (deps - set(keys)) & set(remaining):
                    continue          # a guard reads a call another region still has to answer
                known = {d: _to_pylist(self.ai_values[d]) for d in deps - set(keys) if d in self.ai_values}
                for k in keys:
                    bound[k].guard = G.fold(bound[k].guard, known, n)
                self._run_group(rel, _in_dependency_order(keys, bound))
                remaining = [k for k in remaining if k not in keys]
                ran = True
            if not ran:
                # guards that read each other across regions: ask those calls everywhere
                for k in remaining:
                    bound[k].guard = None

    def _fill_unasked(self, rel: Relation, k: str, node, guard) -> None:
        """A call some earlier clause asked on part of `rel`'s rows (under its own guard): ask it
        on the rows it skipped that `guard` may now need, and merge those answers in."""
        from quail_b200.sql import guards as G
        asked = self.asked_rows.get(k)
        if asked is None or asked.all():
            return
        g = None if guard["op"] == "true" else guard
        if g is not None:
            deps = G.calls_of(g)
            g = G.fold(g, {d: _to_pylist(self.ai_values[d]) for d in deps if d in self.ai_values}, rel.num_rows)
        miss = [r for r in np.nonzero(~asked)[0].tolist() if g is None or G.may_ask(g, r)]
        if not miss:
            return
        saved, saved_asked = self.ai_values, self.asked_rows
        self.ai_values, self.asked_rows = {}, {}
        b = bind_call(node, self.turn, self.model)
        b.drops = False
        self._run_group(rel.take(pa.array(miss, pa.int64())), [b])
        got = self.ai_values
        self.ai_values, self.asked_rows = saved, saved_asked
        for key in (k, k + "#probs"):
            if key not in got or key not in self.ai_values:
                continue
            merged = self.ai_values[key].to_pylist()
            for j, r in enumerate(miss):
                merged[r] = got[key][j].as_py()
            self.ai_values[key] = pa.array(merged, self.ai_values[key].type)
        asked = asked.copy()
        asked[miss] = True
        self.asked_rows[k] = asked

    def _run_group(self, rel: Relation, cs: list[BoundCall]) -> None:
        """One region: the calls `cs` (dependency order) over the rows any of them may be asked on."""
        from quail_b200.sql import guards as G
        n = rel.num_rows
        rows = [r for r in range(n) if any(c.guard is None or G.may_ask(c.guard, r) for c in cs)]
        docs_all = _documents(self.eval(cs[0].doc_expr, rel), n) if n else []
        docs = [docs_all[r] for r in rows]
        expanded = []
        for c in cs:
            guard = None if c.guard is None else G.take(c.guard, rows)
            if c.kind == "extract":
                for qi, q in enumerate(c.questions):
                    bp = (P.bind_d1_read_prompt(q, self.turn) if self.model.layout == "d1"
                          else P.bind_extract_prompt(q, self.turn))
                    stop = None
                    if c.stop is not None and c.fields is not None and c.fields[qi] == c.stop.get("field"):
                        stop = {**c.stop, "call": c.key}
                    expanded.append(BoundCall(key=f"{c.key}#{qi}", kind="extract", preamble=bp.preamble,
                                              tail=bp.tail, doc_expr=c.doc_expr, max_tokens=c.max_tokens,
                                              drops=False, guard=guard, stop=stop))
            else:
                expanded.append(BoundCall(**{**c.__dict__, "guard": guard}))
        got = self._engine_region(cs[0].preamble, docs, expanded) if docs else []
        vals = [{} for _ in range(n)]
        for j, r in enumerate(rows):
            vals[r] = got[j]
        self._store(cs, vals, docs_all)

    def _store(self, cs: list[BoundCall], vals: list[dict], docs_all: list) -> None:
        """Typed Arrow values of calls `cs` from per-row answer dicts (None where not asked)."""
        for c in cs:
            first = f"{c.key}#0" if c.kind == "extract" else c.key
            self.asked_rows[c.key] = np.array([first in v for v in vals], dtype=bool)
            if c.kind == "extract":
                out = []
                for r, v in enumerate(vals):
                    if f"{c.key}#0" not in v:
                        out.append(None)
                        continue
                    answers = [_clean_phrase(v.get(f"{c.key}#{qi}")) for qi in range(len(c.questions))]
                    if c.span:
                        doc = "" if docs_all[r] is None else str(docs_all[r])
                        answers = [_span(doc, a) for a in answers]
                    out.append(answers if c.fields is None else dict(zip(c.fields, answers)))
                item = pa.struct([("start", pa.int64()), ("end", pa.int64())]) if c.span else pa.string()
                typ = pa.list_(item) if c.fields is None else pa.struct([(f, item) for f in c.fields])
                self.ai_values[c.key] = pa.array(out, typ)
            elif c.kind == "classify" and c.probabilities:
                self.ai_values[c.key] = pa.array([v.get(c.key) for v in vals], pa.string())
                self.ai_values[c.key + "#probs"] = pa.array([v.get(c.key + "#probs") for v in vals],
                                                            pa.list_(pa.float64()))
            elif c.kind == "features":
                self.ai_values[c.key] = pa.array(
                    [None if v.get(c.key) is None else [{"feature": f, "strength": x} for f, x in v[c.key]]
                     for v in vals], FEATURE_LIST)
            else:
                typ = {"filter": pa.bool_(), "score": pa.float64(), "classify": pa.string(),
                       "map": pa.string()}[c.kind]
                self.ai_values[c.key] = pa.array([v.get(c.key) for v in vals], typ)

    def _engine_region(self, preamble: str, docs: list, calls: list[BoundCall]) -> list[dict]:
        if self.engine is None:
            raise QueryError("this query needs a model; the session has none")
        from quail_b200.api.engine import CallSpec
        specs = [CallSpec(kind=c.kind, tail=c.tail, name=c.key, labels=c.labels, max_tokens=c.max_tokens,
                          probabilities=c.probabilities, pooling=c.pooling, segments=c.segments, read=c.read,
                          letters=c.letters, drops=c.drops, guard=c.guard, stop=_stop_test(c),
                          stop_when_true=bool(c.stop and c.stop["when_true"] and c.kind == "map"))
                 for c in calls]
        out = self.engine.run_region(preamble, docs, specs)
        self._record(out.stats, "quail.region[" + ",".join(c.kind for c in calls) + "]")
        return out.values

    def _record(self, stats: dict, kind: str) -> None:
        """A model region's stats into the query report: totals, and its metrics under a node id."""
        from quail_b200.runtime.report import node_metrics
        self.report["regions"].append(stats)
        for k in ("asked", "fresh_tokens", "passes"):
            self.report[k] += stats.get(k, 0)
        if stats.get("stopped_early"):
            self.report["stopped_early"] = self.report.get("stopped_early", 0) + stats["stopped_early"]
        self.report["evaluated_documents"] += stats.get("documents", 0)
        nodes = self.report.setdefault("node_metrics", {})
        nodes[f"{len(nodes)}:{kind}"] = node_metrics(stats)

    # ------------------------------------------------------------ SELECT
    def select(self, node) -> pa.Table:
        plan = self._slice_plan(node)
        if plan is not None:
            parts = list(self.select_slices(node, plan))
            return pa.concat_tables(parts) if len(parts) > 1 else parts[0]
        return self._select_whole(node)

    # ------------------------------------------------------------ fetch demand and streaming
    def _slice_plan(self, node):
        """How a SELECT can run slice by slice, or None when it needs all its rows at once.

        It can when it has no aggregate, GROUP BY, HAVING or DISTINCT, and its
        ORDER BY keys (if any) read no model call: the rows are then sorted
        before any model call, so each slice's output is final.
        """
        if "from" not in node or node.get("having") or node.get("group_by"):
            return None
        if node.get("distinct") and not self._distinct_keeps_every_row(node):
            return None
        items = node["items"]
        if any(is_aggregate(n) for it in items for n in walk(it["expr"])):
            return None
        order = []
        for o in node.get("order_by", []):
            e = o["expr"]
            if e.get("type") == "literal" and e.get("kind") == "int":
                e = items[int(e["value"]) - 1]["expr"]
            elif e.get("type") == "column" and e.get("table") is None:
                for it in items:
                    if (it.get("alias") or "").lower() == e["name"].lower():
                        e = it["expr"]
                        break
            if e.get("type") == "star" or has_model_call(e):
                return None
            order.append((e, o["desc"]))
        off = int(literal_value(node["offset"])) if node.get("offset") else 0
        lim = int(literal_value(node["limit"])) if node.get("limit") is not None else None
        return {"order": order, "offset": off, "limit": lim}

    def _distinct_keeps_every_row(self, node) -> bool:
        """A DISTINCT over one table's rows whose SELECT list includes that table's key (a
        DocumentProvider's id column, or *) removes no row, so it needs no whole-table pass and
        a LIMIT above it reaches the model calls below. Reference:
        crates/quail-datafusion/src/rules/distinct.rs."""
        frm = node.get("from") or []
        if len(frm) != 1 or node.get("joins") or frm[0].get("type") != "table":
            return False
        name = frm[0]["name"].lower()
        if name in self.ctes:
            return False
        prov = next((p for k, p in self.catalog.items() if k.lower() == name), None)
        key = getattr(prov, "id_col", None)
        if key is None:
            return False
        alias = (frm[0].get("alias") or frm[0]["name"]).lower()
        for it in node["items"]:
            e = it["expr"]
            if e.get("type") == "star" and e.get("table") in (None, alias, name):
                return True
            if (e.get("type") == "column" and e["name"].lower() == key.lower()
                    and (e.get("table") or alias).lower() in (alias, name)):
                return True
        return False

    def _filter_selectivity(self, ai: list) -> float:
        est = 1.0
        for c in ai:
            inner = c["args"][0] if c.get("type") == "call" and c["name"] == "HINT" else c
            sel = None
            if is_model_call(inner) and inner["name"] in ("AI.IF", "AI_FILTER"):
                sel = bind_call(inner, self.turn, self.model).selectivity
            est *= 0.5 if sel is None else max(float(sel), 0.01)
        return est

    def select_slices(self, node, plan: dict, *, stream_rows: int | None = None, extra_limit: int | None = None):
        """Run a sliceable SELECT; yield its output a slice of input rows at a time.

        With a LIMIT (or `extra_limit`) and demand rules on, rows go to the
        model in slices sized from the pass rate seen so far, and no slice is
        asked once enough rows came through (the fetch demand). With
        `stream_rows`, slices start at that many rows and double, so the first
        rows come back early. Otherwise one slice holds every row.
        """
        rel = self.from_clause(node)
        where = node.get("where")
        plain = [c for c in conjuncts(where) if not has_model_call(c)]
        ai = [c for c in conjuncts(where) if has_model_call(c)]
        for c in plain:
            rel = rel.filter(_as_mask(self.eval(c, rel)))
        if plan["order"]:
            tmp = rel.table
            keys = []
            for k, (e, desc) in enumerate(plan["order"]):
                tmp = tmp.append_column(f"__order{k}", _as_array(self.eval(e, rel), rel.num_rows))
                keys.append((f"__order{k}", "descending" if desc else "ascending"))
            rel = rel.take(pc.sort_indices(tmp, sort_keys=keys, null_placement="at_end"))
        off, lim = plan["offset"], plan["limit"]
        if extra_limit is not None:
            lim = extra_limit if lim is None else min(lim, extra_limit)
        need = None if lim is None else off + lim
        n = rel.num_rows
        fetch = self.pushdown and need is not None and bool(ai) or stream_rows is not None
        sel = self._filter_selectivity(ai)
        start = emitted = tried = passed = 0
        first = True
        size_hint = stream_rows
        while first or (start < n and (need is None or emitted < need)):
            size = n - start
            if fetch and need is not None and self.pushdown and ai:
                rate = (passed + 1) / (tried + 2) if tried else sel
                size = min(size, max(32, int(-(-(need - emitted) * 1.25 // max(rate, 0.02)))))
            if stream_rows is not None:
                size = min(size, size_hint)
                size_hint *= 2
            part = rel.take(pa.array(np.arange(start, start + size, dtype=np.int64))) if size < n else rel
            start += size
            fused = self._filters_with_riders(part, ai, node)
            pre_asked = None
            if fused is not None:
                kept, pre = fused
            else:
                self.carried = ({}, {})
                kept = self.apply_ai_conjuncts(part, ai)
                (pre, pre_asked), self.carried = self.carried, ({}, {})
            tried += part.num_rows
            passed += kept.num_rows
            out = self._project(kept, node, pre, pre_asked)
            lo, hi = emitted, emitted + out.num_rows
            emitted = hi
            a = max(off - lo, 0)
            b = out.num_rows if need is None else max(min(need - lo, out.num_rows), 0)
            if first or b > a:
                yield out.slice(a, max(b - a, 0))
            first = False
            if need is not None and emitted >= need:
                break

    def _filters_with_riders(self, rel: Relation, ai: list, node):
        """WHERE AI.IF chain and the SELECT list's calls on the same document in one region.

        When every model conjunct is an AI.IF over one document (one instruction
        layout), the projection's calls on that document ride in the same region:
        asked as follow-up questions right after the filters kept the row, while
        its document's KV is still resident (the reference runs a chain's
        operators in the same passes, quail/backends/quail/executor/region.py).
        Returns (kept rows, their projection values) or None when it does not apply.
        """
        from quail_b200.planner.search import doc_tokens, order_filters
        from quail_b200.sql import guards as G
        if not ai or rel.num_rows == 0:
            return None
        filters = []
        for c in ai:
            inner = c["args"][0] if c.get("type") == "call" and c["name"] == "HINT" else c
            if not (is_model_call(inner) and inner["name"] in ("AI.IF", "AI_FILTER")):
                return None
            filters.append(bind_call(inner, self.turn, self.model))
        key = (filters[0].preamble, node_key(filters[0].doc_expr))
        if any((f.preamble, node_key(f.doc_expr)) != key for f in filters):
            return None
        demand = G.Demand(self, rel, enabled=self.pushdown)
        for it in node["items"]:
            demand.visit(it["expr"])
        riders = {}
        for k, (call_node, guard) in demand.guards.items():
            b = bind_call(call_node, self.turn, self.model)
            if (b.preamble, node_key(b.doc_expr)) != key or b.kind == "extract":
                continue
            b.drops = False
            b.guard = None if guard["op"] == "true" else guard
            riders[k] = b
        riders = {k: b for k, b in riders.items() if G.calls_of(b.guard) <= set(riders)}
        if not riders:
            return None
        order = order_filters([doc_tokens(b.tail) for b in filters],
                              [b.selectivity if b.selectivity is not None else 0.5 for b in filters])
        chain = [filters[i] for i in order] + _in_dependency_order(list(riders), riders)
        docs = _documents(self.eval(filters[0].doc_expr, rel), rel.num_rows)
        vals = self._engine_region(key[0], docs, chain)
        keep = [all(v.get(f.key, False) for f in filters) for v in vals]
        idx = [i for i, k in enumerate(keep) if k]
        kept = rel.filter(pa.array(keep))
        saved = self.ai_values
        self.ai_values = {}
        self._store(list(riders.values()), [vals[i] for i in idx], [docs[i] for i in idx])
        pre, self.ai_values = self.ai_values, saved
        return kept, pre

    def _project(self, rel: Relation, node, pre: dict | None = None, pre_asked: dict | None = None) -> pa.Table:
        """The SELECT list of a non-aggregating query over `rel` (its model calls asked on demand;
        `pre` holds values some calls already got, aligned with `rel`)."""
        items = node["items"]
        self.ai_values = dict(pre or {})
        self.asked_rows = dict(pre_asked or {})
        self.compute_ai(rel, [it["expr"] for it in items])
        names, arrays = [], []
        unnest = None
        for it in items:
            e = it["expr"]
            if e.get("type") == "call" and e.get("name") == "UNNEST":
                # one row per element of the list; the other items repeat per row
                if unnest is not None or len(e.get("args", [])) != 1:
                    raise QueryError("a SELECT list takes one UNNEST of one list")
                unnest = len(arrays)
                names.append(it.get("alias") or "unnest")
                arrays.append(_as_array(self.eval(e["args"][0], rel), rel.num_rows))
                continue
            if e.get("type") == "star":
                for i, (q, n) in enumerate(rel.cols):
                    if e.get("table") is None or (q or "").lower() == e["table"].lower():
                        if n.startswith("__"):
                            continue
                        names.append(n)
                        arrays.append(rel.column(i))
                continue
            names.append(it.get("alias") or expr_name(e))
            arrays.append(_as_array(self.eval(e, rel), rel.num_rows))
        self.ai_values = {}
        if unnest is not None:
            lst = arrays[unnest]
            if isinstance(lst, pa.ChunkedArray):
                lst = lst.combine_chunks()
            if not pa.types.is_list(lst.type) and not pa.types.is_large_list(lst.type):
                raise QueryError(f"UNNEST takes a list, not {lst.type}")
            parents = pc.list_parent_indices(lst)
            arrays = [pc.list_flatten(lst) if i == unnest else pc.take(a, parents) for i, a in enumerate(arrays)]
        return pa.Table.from_arrays(arrays, names=_dedupe(names))

    def stream(self, tree: dict, batch_rows: int = 65_536, limit: int | None = None):
        """Yield the query's rows as tables, each slice's as soon as its region finishes.

        The first table may be empty; it always comes, so the caller has the schema.
        """
        node = tree
        plan = self._slice_plan(node) if node.get("type") == "select" and not node.get("with") else None
        if plan is None:
            out = self.run(tree)
            yield out if limit is None else out.slice(0, limit)
            return
        yield from self.select_slices(node, plan, stream_rows=min(batch_rows, 1024), extra_limit=limit)

    def _select_whole(self, node) -> pa.Table:
        rel = self.from_clause(node)
        self.carried = ({}, {})
        if node.get("where"):
            rel = self.apply_where(rel, node["where"])
        items = node["items"]
        group_by = node.get("group_by")
        aggregated = group_by is not None or any(is_aggregate(n) for it in items for n in walk(it["expr"]))
        # AI calls in the projection / ORDER BY / HAVING run on the surviving rows (answers the
        # WHERE already got are read, not asked again)
        (self.ai_values, self.asked_rows), self.carried = self.carried, ({}, {})
        ai_exprs = [it["expr"] for it in items] + [o["expr"] for o in node.get("order_by", [])]
        if node.get("having"):
            ai_exprs.append(node["having"])
        self.compute_ai(rel, ai_exprs)
        if aggregated:
            out = self._aggregate(rel, node)
        else:
            names, arrays = [], []
            for it in items:
                e = it["expr"]
                if e.get("type") == "star":
                    for i, (q, n) in enumerate(rel.cols):
                        if e.get("table") is None or (q or "").lower() == e["table"].lower():
                            if n.startswith("__"):
                                continue
                            names.append(n)
                            arrays.append(rel.column(i))
                    continue
                names.append(it.get("alias") or expr_name(e))
                arrays.append(_as_array(self.eval(e, rel), rel.num_rows))
            out = pa.Table.from_arrays(arrays, names=_dedupe(names))
            if node.get("order_by"):
                keys = []
                for k, o in enumerate(node["order_by"]):
                    arr = self._order_key(o["expr"], rel, out, items)
                    out = out.append_column(f"__order{k}", arr)
                    keys.append((f"__order{k}", "descending" if o["desc"] else "ascending"))
                idx = pc.sort_indices(out, sort_keys=keys, null_placement="at_end")
                out = out.take(idx).drop_columns([k for k, _ in keys])
            self.ai_values = {}
            if node.get("distinct"):
                out = _distinct(out)
            return self._limit(out, node)
        self.ai_values = {}
        if node.get("distinct"):
            out = _distinct(out)
        return self._order_limit_output(out, node)

    def _order_key(self, e, rel: Relation, out: pa.Table, items):
        if e.get("type") == "literal" and e["kind"] == "int":
            return out.column(int(e["value"]) - 1)
        if e.get("type") == "column" and e.get("table") is None:
            for it in items:
                if (it.get("alias") or "").lower() == e["name"].lower():
                    return out.column(it["alias"])
        return _as_array(self.eval(e, rel), rel.num_rows)

    def _order_limit_output(self, out: pa.Table, node) -> pa.Table:
        if node.get("order_by"):
            keys = []
            tmp = out
            rel = Relation.from_table(out, None)
            for k, o in enumerate(node["order_by"]):
                e = o["expr"]
                if e.get("type") == "literal" and e["kind"] == "int":
                    arr = out.column(int(e["value"]) - 1)
                else:
                    arr = _as_array(self.eval(e, rel), out.num_rows)
                tmp = tmp.append_column(f"__order{k}", arr)
                keys.append((f"__order{k}", "descending" if o["desc"] else "ascending"))
            idx = pc.sort_indices(tmp, sort_keys=keys, null_placement="at_end")
            out = out.take(idx)
        return self._limit(out, node)

    def _limit(self, out: pa.Table, node) -> pa.Table:
        off = int(literal_value(node["offset"])) if node.get("offset") else 0
        if node.get("limit") is not None:
            return out.slice(off, int(literal_value(node["limit"])))
        return out.slice(off) if off else out

    # ------------------------------------------------------------ aggregates
    def _aggregate(self, rel: Relation, node) -> pa.Table:
        group_by = node.get("group_by") or []
        items = node["items"]
        # resolve GROUP BY ordinal / alias references
        gexprs = []
        for g in group_by:
            if g.get("type") == "literal" and g["kind"] == "int":
                gexprs.append(items[int(g["value"]) - 1]["expr"])
            elif g.get("type") == "column" and g.get("table") is None and any(
                    (it.get("alias") or "").lower() == g["name"].lower() for it in items):
                gexprs.append(next(it["expr"] for it in items if (it.get("alias") or "").lower() == g["name"].lower()))
            else:
                gexprs.append(g)
        aggs = []
        for e in [it["expr"] for it in items] + ([node["having"]] if node.get("having") else []) + \
                [o["expr"] for o in node.get("order_by", [])]:
            for n in walk(e):
                if is_aggregate(n) and node_key(n) not in [node_key(a) for a in aggs]:
                    aggs.append(n)
        cols = {}
        for i, g in enumerate(gexprs):
            cols[f"g{i}"] = _as_array(self.eval(g, rel), rel.num_rows)
        specs = []
        for i, a in enumerate(aggs):
            fn = a["name"]
            args = a["args"]
            if fn == "COUNT" and (not args or args[0].get("type") == "star"):
                cols[f"a{i}"] = pa.array(np.ones(rel.num_rows, dtype=np.int64))
                specs.append((f"a{i}", "count", None))
                continue
            cols[f"a{i}"] = _as_array(self.eval(args[0], rel), rel.num_rows)
            op = {"COUNT": "count_distinct" if a.get("distinct") else "count", "SUM": "sum", "AVG": "mean",
                  "MIN": "min", "MAX": "max", "ARRAY_AGG": "list", "ANY_VALUE": "first"}[fn]
            specs.append((f"a{i}", op, None))
        if not gexprs:
            # one group holding every row (an empty input still gives one row)
            cols["g_all"] = pa.array(np.zeros(rel.num_rows, dtype=np.int64))
        base = pa.table(cols)
        keys = [f"g{i}" for i in range(len(gexprs))] or ["g_all"]
        grouped = base.group_by(keys, use_threads=False).aggregate([(c, op) for c, op, _ in specs])
        rename = {f"{c}_{op}": c for c, op, _ in specs}
        grouped = grouped.rename_columns([rename.get(n, n) for n in grouped.column_names])
        if not gexprs and grouped.num_rows == 0:
            empty = {}
            for c, op, _ in specs:
                empty[c] = pa.array([0 if op in ("count", "count_distinct") else None])
            grouped = pa.table(empty) if empty else pa.table({"g_all": [0]})
        grel = Relation.from_table(grouped, None)
        self._agg_map = {node_key(a): grel.resolve(None, f"a{i}") for i, a in enumerate(aggs)}
        self._group_map = {node_key(g): grel.resolve(None, f"g{i}") for i, g in enumerate(gexprs)}
        if node.get("having"):
            grel = grel.filter(_as_mask(self.eval(node["having"], grel)))
        names, arrays = [], []
        for it in items:
            names.append(it.get("alias") or expr_name(it["expr"]))
            arrays.append(_as_array(self.eval(it["expr"], grel), grel.num_rows))
        out = pa.Table.from_arrays(arrays, names=_dedupe(names))
        if node.get("order_by"):
            keys = []
            for k, o in enumerate(node["order_by"]):
                arr = self._order_key(o["expr"], grel, out, items)
                out = out.append_column(f"__order{k}", arr)
                keys.append((f"__order{k}", "descending" if o["desc"] else "ascending"))
            idx = pc.sort_indices(out, sort_keys=keys, null_placement="at_end")
            out = out.take(idx).drop_columns([k for k, _ in keys])
        self._agg_map, self._group_map = {}, {}
        return out

    # ------------------------------------------------------------ scalar expressions
    def eval(self, e, rel: Relation):
        t = e.get("type")
        k = node_key(e)
        if getattr(self, "_agg_map", None) and k in self._agg_map:
            return rel.column(self._agg_map[k])
        if getattr(self, "_group_map", None) and k in self._group_map:
            return rel.column(self._group_map[k])
        if t == "column":
            return rel.column(rel.resolve(e.get("table"), e["name"]))
        if t == "literal":
            return pa.scalar(e["value"]) if e["value"] is not None else pa.scalar(None, pa.null())
        if t == "binary":
            return self._binary(e, rel)
        if t == "unary":
            v = self.eval(e["arg"], rel)
            return pc.invert(_bool(v)) if e["op"] == "NOT" else pc.negate(v)
        if t == "is_null":
            v = self.eval(e["arg"], rel)
            r = pc.is_null(v)
            return pc.invert(r) if e["negated"] else r
        if t == "is_bool":
            v = _bool(self.eval(e["arg"], rel))
            r = pc.fill_null(pc.equal(v, pa.scalar(e["value"])), False)
            return pc.invert(r) if e["negated"] else r
        if t == "in":
            v = self.eval(e["arg"], rel)
            if "query" in e:
                # IN (SELECT ...): the subquery's single column is the value set
                sub = self.query(e["query"])
                if sub.num_columns != 1:
                    raise QueryError("IN (SELECT ...) needs a subquery of one column")
                vals = sub.column(0).combine_chunks()
            else:
                vals = pa.array([literal_value(x) for x in e["list"]])
            r = pc.fill_null(pc.is_in(_as_array(v, rel.num_rows), value_set=vals), False)
            return pc.invert(r) if e["negated"] else r
        if t == "between":
            v = self.eval(e["arg"], rel)
            r = pc.and_(pc.greater_equal(v, self.eval(e["low"], rel)), pc.less_equal(v, self.eval(e["high"], rel)))
            return pc.invert(r) if e["negated"] else r
        if t == "like":
            v = self.eval(e["arg"], rel)
            pat = literal_value(e["pattern"])
            r = pc.match_like(_as_array(v, rel.num_rows), pat, ignore_case=e.get("case_insensitive", False))
            return pc.invert(r) if e["negated"] else r
        if t == "case":
            return self._case(e, rel)
        if t == "cast":
            return _cast(self.eval(e["arg"], rel), e["to"])
        if t == "array":
            return pa.scalar([literal_value(x) for x in e["items"]])
        if t == "subscript":
            v = _as_array(self.eval(e["arg"], rel), rel.num_rows)
            idx = literal_value(e["index"])
            if isinstance(idx, int):
                return pc.list_element(v, idx)
            return pc.struct_field(v, idx)
        if t == "call":
            return self._call(e, rel)
        if t == "star":
            raise QueryError("* is not an expression here")
        if t == "scalar_subquery":
            sub = self.query(e["query"])
            if sub.num_columns != 1 or sub.num_rows > 1:
                raise QueryError("a scalar subquery returns one value")
            return sub.column(0)[0] if sub.num_rows else pa.scalar(None)
        raise QueryError(f"unsupported expression {t}")

    def _binary(self, e, rel):
        op = e["op"]
        a, b = self.eval(e["left"], rel), self.eval(e["right"], rel)
        if op == "AND":
            return pc.and_kleene(_bool(a), _bool(b))
        if op == "OR":
            return pc.or_kleene(_bool(a), _bool(b))
        if op == "||":
            return pc.binary_join_element_wise(_str(a), _str(b), "")
        fn = {"=": pc.equal, "<>": pc.not_equal, "<": pc.less, "<=": pc.less_equal, ">": pc.greater,
              ">=": pc.greater_equal, "+": pc.add, "-": pc.subtract, "*": pc.multiply, "%": _mod}.get(op)
        if op == "/":
            return pc.divide(_float(a), _float(b))
        if fn is None:
            raise QueryError(f"unsupported operator {op}")
        return fn(a, b)

    def _case(self, e, rel):
        n = rel.num_rows
        result = None
        remaining = pa.array(np.ones(n, dtype=bool))
        operand = self.eval(e["operand"], rel) if e.get("operand") else None
        out_vals = [None] * n
        for cond, val in e["whens"]:
            c = pc.equal(operand, self.eval(cond, rel)) if operand is not None else self.eval(cond, rel)
            c = pc.fill_null(_as_array(_bool(c), n), False)
            take = pc.and_(remaining, c)
            v = _as_array(self.eval(val, rel), n).to_pylist()
            for i, tk in enumerate(take.to_pylist()):
                if tk:
                    out_vals[i] = v[i]
            remaining = pc.and_(remaining, pc.invert(c))
        if e.get("else") is not None:
            v = _as_array(self.eval(e["else"], rel), n).to_pylist()
            for i, r in enumerate(remaining.to_pylist()):
                if r:
                    out_vals[i] = v[i]
        result = pa.array(out_vals)
        return result

    def _call(self, e, rel):
        name = e["name"]
        if is_model_call(e):
            k = node_key(e)
            if k not in self.ai_values:
                self.compute_ai(rel, [e])
            v = self.ai_values[k]
            return v
        if name == "HINT":
            return self.eval(e["args"][0], rel)
        if name == "PROMPT":
            raise QueryError("PROMPT is the input of an AI function, not a value")
        name = CPU_ALIASES.get(name, name)
        if name in CPU_AI_FUNCTIONS:
            from quail_b200.sql import documents
            args = [self.eval(a, rel) for a in e["args"]]
            return documents.call(name, args, rel.num_rows)
        if name == "UNNEST":
            raise QueryError("UNNEST expands a list into rows: it is an item of a SELECT list")
        args = [self.eval(a, rel) for a in e["args"] if a.get("type") != "named_arg"]
        fns = {
            "UPPER": lambda a: pc.utf8_upper(a[0]), "LOWER": lambda a: pc.utf8_lower(a[0]),
            "LENGTH": lambda a: pc.utf8_length(a[0]), "CHAR_LENGTH": lambda a: pc.utf8_length(a[0]),
            "TRIM": lambda a: pc.utf8_trim_whitespace(a[0]), "ABS": lambda a: pc.abs(a[0]),
            "ROUND": lambda a: pc.round(a[0], int(a[1].as_py()) if len(a) > 1 else 0),
            "FLOOR": lambda a: pc.floor(a[0]), "CEIL": lambda a: pc.ceil(a[0]),
            "COALESCE": lambda a: pc.coalesce(*a), "CONCAT": lambda a: pc.binary_join_element_wise(*[_str(x) for x in a], ""),
            "SUBSTR": lambda a: _substr(a), "SUBSTRING": lambda a: _substr(a),
            "LEFT": lambda a: pc.utf8_slice_codeunits(a[0], 0, max(int(a[1].as_py()), 0)),
            "CHARACTER_LENGTH": lambda a: pc.utf8_length(a[0]),
            "STARTS_WITH": lambda a: pc.starts_with(a[0], a[1].as_py()),
            "CONTAINS": lambda a: pc.match_substring(a[0], a[1].as_py()),
            "REGEXP_LIKE": lambda a: pc.match_substring_regex(a[0], a[1].as_py()),
            "ARRAY_LENGTH": lambda a: pc.list_value_length(a[0]),
            "CARDINALITY": lambda a: pc.list_value_length(a[0]),
            "IFF": lambda a: pc.if_else(_bool(a[0]), a[1], a[2]),
            "NULLIF": lambda a: pc.if_else(pc.equal(a[0], a[1]), pa.scalar(None, a[0].type), a[0]),
            "GREATEST": lambda a: pc.max_element_wise(*a), "LEAST": lambda a: pc.min_element_wise(*a),
        }
        if name in fns:
            return fns[name](args)
        raise QueryError(f"unknown function {name}")


# ---------------------------------------------------------------- small helpers

def _in_dependency_order(keys: list, bound: dict) -> list:
    """The calls of one region, each after the calls its guard reads (otherwise as found)."""
    from quail_b200.sql import guards as G
    out, placed = [], set()
    pending = list(keys)
    while pending:
        for k in pending:
            if G.calls_of(bound[k].guard) & set(pending) - {k} <= placed:
                break
        else:
            k = pending[0]            # a cycle cannot come from the rules; keep the order found
        out.append(bound[k])
        placed.add(k)
        pending.remove(k)
    return out


def _as_array(v, n):
    if isinstance(v, pa.Scalar):
        return pa.array([v.as_py()] * n, type=v.type if v.type != pa.null() else None)
    if isinstance(v, pa.ChunkedArray):
        return v.combine_chunks() if v.num_chunks != 1 else v.chunk(0)
    return v


def _as_mask(v):
    if isinstance(v, pa.Scalar):
        return v.as_py() is True
    return pc.fill_null(_bool(v), False)


def _bool(v):
    t = v.type
    if t == pa.bool_():
        return v
    if t == pa.null():
        return pc.cast(v, pa.bool_()) if not isinstance(v, pa.Scalar) else pa.scalar(None, pa.bool_())
    return pc.cast(v, pa.bool_())


def _str(v):
    return pc.cast(v, pa.string()) if v.type != pa.string() else v


def _float(v):
    return pc.cast(v, pa.float64()) if not pa.types.is_floating(v.type) else v


def _mod(a, b):
    return pc.subtract(a, pc.multiply(pc.floor(pc.divide(_float(a), _float(b))).cast(pa.int64()), b))


def _substr(a):
    start = int(a[1].as_py()) - 1
    if len(a) > 2:
        return pc.utf8_slice_codeunits(a[0], start, start + int(a[2].as_py()))
    return pc.utf8_slice_codeunits(a[0], start)


def _cast(v, to: str):
    base = to.split("(")[0]
    typ = {"INT": pa.int64(), "INTEGER": pa.int64(), "BIGINT": pa.int64(), "FLOAT": pa.float64(),
           "DOUBLE": pa.float64(), "REAL": pa.float32(), "DECIMAL": pa.float64(), "NUMBER": pa.float64(),
           "VARCHAR": pa.string(), "STRING": pa.string(), "TEXT": pa.string(), "BOOLEAN": pa.bool_(),
           "BOOL": pa.bool_(), "DATE": pa.date32(), "TIMESTAMP": pa.timestamp("us")}.get(base)
    if typ is None:
        raise QueryError(f"unsupported CAST type {to}")
    return pc.cast(v, typ)


def _dedupe(names):
    seen, out = {}, []
    for n in names:
        if n in seen:
            seen[n] += 1
            out.append(f"{n}_{seen[n]}")
        else:
            seen[n] = 0
            out.append(n)
    return out


def _distinct(t: pa.Table) -> pa.Table:
    if t.num_rows == 0:
        return t
    rows = {}
    for i, r in enumerate(zip(*[c.to_pylist() for c in t.columns])):
        key = json.dumps(r, default=str)
        rows.setdefault(key, i)
    return t.take(pa.array(sorted(rows.values())))


def _documents(v, n: int) -> list:
    """Each row's document: a string, or for a list<int> column (token ids) a numpy view of
    the row's ids (no Python list per row: the engine takes arrays as they are)."""
    if isinstance(v, pa.Scalar):
        return [v.as_py()] * n
    arr = v.combine_chunks() if isinstance(v, pa.ChunkedArray) else v
    if pa.types.is_list(arr.type) or pa.types.is_large_list(arr.type):
        if pa.types.is_integer(arr.type.value_type) and arr.null_count == 0:
            flat = arr.values.to_numpy(zero_copy_only=False).astype(np.int32, copy=False)
            offs = arr.offsets.to_numpy()
            return [flat[offs[i]:offs[i + 1]] for i in range(len(arr))]
    return arr.to_pylist()


def _to_pylist(v):
    if isinstance(v, pa.Scalar):
        return v.as_py()
    return v.to_pylist()


def _stop_test(c: BoundCall):
    """text so far -> decision of the WHERE test of call c's answer (quail_b200.sql.partial), or
    None. A map answer is its text; an extraction answer one field of its struct, which may still
    be NULL (found nothing), so it is only ever decided NOT TRUE."""
    from quail_b200.sql import partial
    if c.stop is None:
        return None
    test = c.stop["test"]
    if c.kind == "map":
        return lambda text: partial.decide(test, c.key, partial.Completions(text), node_key)
    if c.kind == "extract" and c.stop.get("field") is not None:
        call, field = c.stop["call"], c.stop["field"]

        def decide(text):
            prefix = partial.extraction_prefix(text)
            if prefix is None:
                return partial.UNDECIDED
            return partial.decide(test, call, partial.Completions(prefix, may_be_null=True), node_key, field)
        return decide
    return None


def _clean_phrase(text):
    if text is None:
        return None
    s = str(text).strip()
    if s.lower().startswith("phrase:"):
        s = s[7:].strip()
    return s or None


def _span(doc: str, answer):
    if not answer:
        return None
    i = doc.find(answer)
    return None if i < 0 else {"start": i, "end": i + len(answer)}
