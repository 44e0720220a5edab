"""The client of Quail Server: Arrow Flight calls, and the remote side of a Session.

`ServerClient` wraps the server's calls. `Session(config, endpoint=...)`
uses `RemoteConnection` (tables upload to the server) and `session.sql()`
returns a `RemoteQuery`, whose `submit()` gives a `QueryRun`.

Reference surface: quail/remote/client.py (QueryStatus, QueryFailedError,
ServerClient, QueryRun, RemoteConnection, RemoteQuery).
"""

from __future__ import annotations

import json
import os
from collections.abc import Iterator
from dataclasses import dataclass, fields

import pyarrow as pa
import pyarrow.flight as flight

TOKEN_VARIABLE = "QUAIL_SERVER_TOKEN"
FINISHED_STATES = frozenset({"succeeded", "failed", "cancelled"})
DEFAULT_WAIT_S = 1.0


@dataclass(frozen=True)
class QueryStatus:
    """A submission's status as the server saved it."""

    id: str
    sql: str
    state: str                       # queued | running | succeeded | failed | cancelled
    dialect: str | None = None
    error: str | None = None
    timeout_s: float | None = None
    submitted_at: float | None = None
    started_at: float | None = None
    finished_at: float | None = None
    num_rows: int | None = None
    progress: list | None = None
    revision: int = 0
    plans: tuple = ()
    ready: bool = False
    num_answers: int = 0
    tables: tuple = ()

    @property
    def done(self) -> bool:
        return self.state in FINISHED_STATES

    @classmethod
    def parse(cls, body: bytes) -> "QueryStatus":
        found = json.loads(body)
        known = {f.name for f in fields(cls)}
        kw = {k: v for k, v in found.items() if k in known}
        for k in ("plans", "tables"):
            if k in kw and isinstance(kw[k], list):
                kw[k] = tuple(kw[k])
        return cls(**kw)


class QueryFailedError(RuntimeError):
    """The submission finished without rows (failed or cancelled)."""

    def __init__(self, status: QueryStatus):
        self.status = status
        super().__init__(f"query {status.id} {status.state}: {status.error or status.state}")


class ServerClient:
    def __init__(self, endpoint: str, token: str | None = None):
        self.endpoint = endpoint
        self._flight = flight.FlightClient(endpoint)
        token = token if token is not None else os.environ.get(TOKEN_VARIABLE)
        headers = [(b"authorization", f"Bearer {token}".encode())] if token else []
        self._options = flight.FlightCallOptions(headers=headers)

    def close(self) -> None:
        self._flight.close()

    def _act(self, name: str, body) -> bytes:
        text = body if isinstance(body, str) else json.dumps(body)
        results = list(self._flight.do_action(flight.Action(name, text.encode()), self._options))
        return results[0].body.to_pybytes()

    def upload(self, name: str, table, id_col: str | None = None) -> None:
        """Register rows (a Table or a RecordBatchReader) on the server as table `name`."""
        reader = table if isinstance(table, pa.RecordBatchReader) else pa.RecordBatchReader.from_batches(
            table.schema, table.to_batches())
        path = (name, id_col) if id_col else (name,)
        writer, _ = self._flight.do_put(flight.FlightDescriptor.for_path(*path), reader.schema, self._options)
        try:
            for batch in reader:
                writer.write_batch(batch)
        finally:
            writer.close()

    def submit(self, sql: str, *, dialect: str | None = None, query_id: str | None = None,
               timeout_s: float | None = None) -> QueryStatus:
        asked = {"sql": sql, "dialect": dialect, "id": query_id, "timeout_s": timeout_s}
        return QueryStatus.parse(self._act("submit", {k: v for k, v in asked.items() if v is not None}))

    def status(self, query_id: str, *, after: int | None = None, wait_s: float = 0.0) -> QueryStatus:
        if after is None:
            return QueryStatus.parse(self._act("status", query_id))
        return QueryStatus.parse(self._act("status", {"id": query_id, "after": after, "wait_s": wait_s}))

    def answers(self, query_id: str, *, after: int = 0, limit: int = 1000) -> dict:
        return json.loads(self._act("answers", {"id": query_id, "after": after, "limit": limit}))

    def report(self, query_id: str) -> list:
        return json.loads(self._act("report", query_id))["regions"]

    def cancel(self, query_id: str) -> QueryStatus:
        return QueryStatus.parse(self._act("cancel", query_id))

    def submissions(self) -> list[QueryStatus]:
        return [QueryStatus.parse(json.dumps(s).encode()) for s in json.loads(self._act("list", ""))]

    def explain(self, sql: str, dialect: str | None = None) -> str:
        asked = {"sql": sql} if dialect is None else {"sql": sql, "dialect": dialect}
        return self._act("explain", asked).decode()

    def result_batches(self, query_id: str) -> pa.RecordBatchReader:
        ticket = flight.Ticket(json.dumps({"query_id": query_id}).encode())
        return self._flight.do_get(ticket, self._options).to_reader()

    def stream_batches(self, query_id: str) -> pa.RecordBatchReader:
        ticket = flight.Ticket(json.dumps({"query_id": query_id, "stream": True}).encode())
        return self._flight.do_get(ticket, self._options).to_reader()

    def sql(self, text: str) -> pa.Table:
        """Run a query at once (not queued) and return its rows."""
        return self._flight.do_get(flight.Ticket(text.encode()), self._options).read_all()


class QueryRun:
    """One submission: its status, and its rows once it succeeded."""

    def __init__(self, client: ServerClient, query_id: str):
        self._client = client
        self.id = query_id

    def __repr__(self) -> str:
        return f"QueryRun({self.id!r})"

    def status(self) -> QueryStatus:
        return self._client.status(self.id)

    def watch(self, wait_s: float = DEFAULT_WAIT_S) -> Iterator[QueryStatus]:
        st = self.status()
        while True:
            yield st
            if st.done:
                return
            st = self._client.status(self.id, after=st.revision, wait_s=wait_s)

    def wait(self, wait_s: float = DEFAULT_WAIT_S) -> QueryStatus:
        st = None
        for st in self.watch(wait_s):
            pass
        return st

    def cancel(self) -> QueryStatus:
        return self._client.cancel(self.id)

    def answers(self, after: int = 0, limit: int = 1000) -> dict:
        return self._client.answers(self.id, after=after, limit=limit)

    def report(self) -> list:
        return self._client.report(self.id)

    def stream_result(self, wait_s: float = DEFAULT_WAIT_S) -> pa.RecordBatchReader:
        st = self.wait(wait_s)
        if st.state != "succeeded":
            raise QueryFailedError(st)
        return self._client.result_batches(self.id)

    def result(self, wait_s: float = DEFAULT_WAIT_S):
        from quail_b200.api.session import QueryResult
        st = self.wait(wait_s)
        if st.state != "succeeded":
            raise QueryFailedError(st)
        table = self._client.result_batches(self.id).read_all()
        return QueryResult(table=table, report={"regions": self._client.report(self.id)},
                           plan="\n".join(p.get("text", "") for p in st.plans))


class RemoteConnection:
    """A remote session's connection: its tables and queries live on one server."""

    def __init__(self, endpoint: str, token: str | None = None):
        self.client = ServerClient(endpoint, token)

    def register(self, name: str, provider) -> None:
        from quail_b200.catalog.providers import ScanRequest, as_provider
        p = as_provider(provider)
        table = p.scan(ScanRequest()) if hasattr(p, "scan") else p
        if isinstance(table, pa.RecordBatchReader):
            table = table.read_all()
        self.client.upload(name, table, getattr(p, "id_col", None))

    def run(self, query_id: str) -> QueryRun:
        return QueryRun(self.client, query_id)

    def close(self) -> None:
        self.client.close()


class RemoteQuery:
    """A SQL query that the server plans and runs."""

    def __init__(self, session, text: str, dialect: str = "snowflake"):
        self.session = session
        self.text = text
        self.dialect = dialect

    @property
    def _client(self) -> ServerClient:
        return self.session._remote.client

    def submit(self, *, query_id: str | None = None, timeout_s: float | None = None) -> QueryRun:
        st = self._client.submit(self.text, dialect=self.dialect, query_id=query_id, timeout_s=timeout_s)
        return QueryRun(self._client, st.id)

    def run(self, plan=None, *, timeout_s: float | None = None):
        if plan is not None:
            raise ValueError("a remote query runs the server's plan")
        return self.submit(timeout_s=timeout_s).result()

    def collect(self, limit: int | None = None) -> pa.Table:
        t = self.run().table
        return t if limit is None else t.slice(0, limit)

    def execute_stream(self, batch_rows: int = 65_536, limit: int | None = None, *,
                       timeout_s: float | None = None) -> pa.RecordBatchReader:
        if batch_rows <= 0:
            raise ValueError("batch_rows must be positive")
        if limit is not None and limit < 0:
            raise ValueError("limit must be nonnegative")
        run = self.submit(timeout_s=timeout_s)
        t = self._client.stream_batches(run.id).read_all()
        if limit is not None:
            t = t.slice(0, limit)
        return pa.RecordBatchReader.from_batches(t.schema, t.to_batches(max_chunksize=batch_rows))

    def explain(self, **_options) -> str:
        return self._client.explain(self.text, self.dialect)

    def plan(self):
        raise RuntimeError("a remote query is planned on the server; call explain()")
