"""Session, Query and QueryResult: the public query API.

    config = EngineConfig(model="qwen3-4b-fp8", device="b200")
    with Session(config=config) as session:
        session.register("reviews", DocumentProvider.from_table(reviews, id_col="id"))
        table = session.sql("SELECT r.id FROM reviews r WHERE AI.IF(PROMPT('... {0}', r.body))").collect()

Same surface as the reference (quail/api/session.py:22-232, query.py:102-333,
execution/result.py:312-439): register / register_parquet / register_json /
register_csv, sql() returning a Query with run / collect / execute_stream /
explain / plan, and a QueryResult holding the table, a report of the model
work (fresh tokens, documents, passes, wall time) and the plan text. With
`endpoint=` the session talks to a Quail server instead
(quail_b200.server.client, quail_b200.server.service).
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, field

import pyarrow as pa

from quail_b200.api.config import EngineConfig, check_config
from quail_b200.catalog.providers import ArrowDatasetProvider, as_provider


@dataclass
class QueryResult:
    table: pa.Table
    report: dict = field(default_factory=dict)
    plan: str = ""

    def collect(self) -> pa.Table:
        return self.table

    def explain(self) -> str:
        """The plan with its estimates and, below, what the run measured."""
        return self.plan

    def __repr__(self) -> str:
        return f"QueryResult({self.table.num_rows} rows, {self.report.get('wall_s', 0):.3f} s)"


def _finish_report(rep: dict, session, wall: float) -> None:
    """Whole-query metrics (crates/quail/src/report.rs:355-380): the nodes' summed counts,
    the largest GPU peak in GiB, and the price of the GPU time at the device's hourly rate."""
    from quail_b200.runtime.report import totals
    nodes = rep.setdefault("node_metrics", {})
    tot = totals(nodes)
    rep["cached_tokens"] = tot["cached_tokens"]
    rep["evaluated_document_pairs"] = tot["evaluated_document_pairs"]
    rep["peak_gib"] = tot["peak_gpu_bytes"] / 2 ** 30
    price = None
    cfg = session.config
    if cfg is not None:
        from quail_b200.planner.specs import DEVICES
        dev = DEVICES.get(cfg.device)
        if dev is not None and dev.usd_per_hour:
            price = dev.usd_per_hour
    rep["usd_per_query"] = (wall / 3600.0 * max(cfg.gpus, 1) * price) if price else None
    nodes["output"] = {"output_rows": rep.get("output_rows", 0), "wall_s": wall}


class Query:
    def __init__(self, session: "Session", text: str, dialect: str | None = None):
        from quail_b200.api.dialects import SQLDialect, to_parser_sql
        from quail_b200.sql.executor import parse
        self.session = session
        self.text = text
        if dialect is None:
            dialect = session.settings.get("datafusion.sql_parser.dialect", "snowflake")
        self.dialect = SQLDialect.of(dialect).value
        self.tree = parse(to_parser_sql(text, self.dialect))  # syntax errors surface here, before model work
        if session.registry is not None:
            self.tree = session.registry.apply_rules(self.tree)

    def plan(self):
        from quail_b200.planner.plan import plan_query
        return plan_query(self.tree, self.session)

    def explain(self, *, verbose: bool = False, analyze: bool = False) -> str:
        plan = self.plan()
        text = plan.explain(verbose=verbose)
        if analyze:
            result = self.run()
            text += "\n" + plan.explain_measured(result.report)
        return text

    def run(self) -> QueryResult:
        from quail_b200.sql.executor import Executor
        s = self.session
        t0 = time.perf_counter()
        engine = s.engine() if s._needs_model(self.tree) else None
        boot = time.perf_counter() - t0
        ex = Executor(s.catalog, engine, settings=s.settings)
        t1 = time.perf_counter()
        if self.tree.get("type") == "set":
            s.settings[self.tree["name"]] = self.tree["value"].get("value")
            table = pa.table({"ok": [True]})
        else:
            table = ex.run(self.tree if self.tree.get("type") != "explain" else self.tree["query"])
        wall = time.perf_counter() - t1
        rep = dict(ex.report)
        rep.update(wall_s=wall, boot_s=boot, output_rows=table.num_rows)
        rep["documents_per_second"] = rep["evaluated_documents"] / wall if wall > 0 else 0.0
        _finish_report(rep, s, wall)
        plan = self.plan()
        text = plan.explain() if self.tree.get("type") == "set" else plan.explain() + "\n" + plan.explain_measured(rep)
        return QueryResult(table=table, report=rep, plan=text)

    def collect(self, limit: int | None = None) -> pa.Table:
        t = self.run().table
        return t if limit is None else t.slice(0, limit)

    def execute_stream(self, batch_rows: int = 65_536, limit: int | None = None):
        """The rows as a RecordBatchReader that yields each slice's rows once its region finished.

        A query that can run slice by slice (no aggregate, DISTINCT, or ORDER BY on a
        model answer) sends its first rows to the model in a small slice and
        doubles the slice each time, so rows arrive while later ones are asked; a
        limit stops asking once enough rows came through. Other queries return
        their rows when the whole query finished (reference: crates/quail/src/lib.rs:376).
        """
        from quail_b200.sql.executor import Executor
        if batch_rows < 1:
            raise ValueError(f"batch_rows={batch_rows}: at least one row per batch")
        if limit is not None and limit < 0:
            raise ValueError(f"limit={limit}: a row limit cannot be negative")
        s = self.session
        engine = s.engine() if s._needs_model(self.tree) else None
        ex = Executor(s.catalog, engine, settings=s.settings)
        parts = ex.stream(self.tree, batch_rows, limit)
        first = next(parts)

        def batches():
            yield from first.to_batches(max_chunksize=batch_rows)
            for part in parts:
                yield from part.cast(first.schema).to_batches(max_chunksize=batch_rows)

        return pa.RecordBatchReader.from_batches(first.schema, batches())

    def submit(self, **options):
        raise RuntimeError("submit() sends a query to a Quail server; this session has no endpoint")


class Session:
    def __init__(self, config: EngineConfig | None = None, *, tokenizer=None, registry=None,
                 endpoint: str | None = None, token: str | None = None):
        self.config = config
        self.registry = registry     # quail_b200.extensions.ExtensionRegistry: extra models, devices, rules
        self.model_cfg = check_config(config, registry) if config is not None else None
        self.catalog: dict = {}
        self.settings: dict = {}
        self.tokenizer_path = tokenizer
        self._engine = None
        self._remote = None
        if endpoint is not None:
            from quail_b200.server.client import RemoteConnection
            self._remote = RemoteConnection(endpoint, token)

    # ------------------------------------------------------------ tables
    def register(self, name: str, provider) -> None:
        if self._remote is not None:
            self._remote.register(name, provider)
            return
        self.catalog[name] = as_provider(provider)

    def register_parquet(self, name: str, path: str) -> None:
        self.register(name, ArrowDatasetProvider(path, "parquet"))

    def register_csv(self, name: str, path: str) -> None:
        self.register(name, ArrowDatasetProvider(path, "csv"))

    def register_json(self, name: str, path: str) -> None:
        self.register(name, ArrowDatasetProvider(path, "json"))

    def deregister(self, name: str) -> None:
        self.catalog.pop(name, None)

    # ------------------------------------------------------------ queries
    def sql(self, text: str, dialect: str | None = None):
        """A query in `dialect` (quail_b200.SQLDialect: 'snowflake', the default, or 'bq')."""
        if self._remote is not None:
            from quail_b200.server.client import RemoteQuery
            return RemoteQuery(self, text, dialect or "snowflake")
        return Query(self, text, dialect)

    def get_run(self, query_id: str):
        """The run of a query a server already has (remote sessions)."""
        if self._remote is None:
            raise RuntimeError("get_run() reads a Quail server's submission; this session has no endpoint")
        return self._remote.run(query_id)

    def _needs_model(self, tree) -> bool:
        from quail_b200.sql.executor import has_model_call
        return has_model_call(tree)

    def attach_engine(self, engine) -> None:
        """Use an already started engine (a replica loaded elsewhere in this process)."""
        self._engine = engine

    def engine(self):
        """The model engine (started on first use: weights loaded, arena sized)."""
        if self._engine is None:
            factory = (self.registry.backend(self.config.backend)
                       if self.config.backend != "quail" and self.registry is not None else None)
            if factory is not None:
                # a comparison backend (quail_b200.baselines): the same SQL, another engine
                self._engine = factory(self.config, self.registry)
                return self._engine
            if self.config.gpus > 1:
                from quail_b200.runtime.workers import WorkerPool
                self._engine = WorkerPool(self.config, registry=self.registry)
            else:
                from quail_b200.api.engine import ModelEngine
                from quail_b200.engine.token_store import TokenStore
                self._engine = ModelEngine(self.config, registry=self.registry)
                # documents tokenized once per session (QUAIL_TOKEN_STORE_TOKENS caps it)
                cap = int(os.environ.get("QUAIL_TOKEN_STORE_TOKENS", "200000000"))
                self._engine.token_store = TokenStore(cap) if cap > 0 else None
        return self._engine

    def interrupt(self) -> None:
        """Stop the model work of this session now: a running query fails, and queries fail at
        once until resume() (crates/quail/src/lib.rs:265-273). Worker processes are killed and
        come back, models reloaded, on the first query after resume()."""
        eng = self._engine
        if eng is None:
            return
        if hasattr(eng, "interrupt") and callable(eng.interrupt):
            eng.interrupt()
        else:
            import threading
            flag = getattr(eng, "interrupt", None)
            if not isinstance(flag, threading.Event):
                eng.interrupt = threading.Event()
            eng.interrupt.set()

    def resume(self) -> None:
        eng = self._engine
        if eng is None:
            return
        if hasattr(eng, "resume"):
            eng.resume()
        elif getattr(eng, "interrupt", None) is not None:
            eng.interrupt.clear()

    def close(self) -> None:
        if self._engine is not None:
            self._engine.close()
            self._engine = None
        if self._remote is not None:
            self._remote.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def run_filter_query(pipe, arena, workload, *, chunk_tokens: int = 16384, name: str = "if"):
    """Run `SELECT ... WHERE AI.IF(PROMPT(<instruction> {0}, body))` over a token table.

    `workload` holds the tokenized template prefix, the question suffix and
    one body per row (the benchmark's synthetic table); this is the region a
    session runs for that query, on an already loaded replica. Returns the
    kept row indices and executor stats.
    """
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor

    rows = getattr(pipe, "w", pipe).answer_rows.shape[0]
    half = rows // 2
    ex = StageExecutor(pipe, arena, chunk_tokens)
    call = Call(kind="filter", suffix=workload.suffix, true_cols=list(range(half)),
                false_cols=list(range(half, rows)), name=name)
    results = RegionRun(ex, workload.prefix, workload.bodies, [call]).run()
    kept = [i for i, r in enumerate(results) if r.values.get(name)]
    return {"kept": kept, "stats": ex.stats, "results": results}
