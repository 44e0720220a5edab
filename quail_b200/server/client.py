"""Client side of Quail Server, and the remote flavour of a Session.

Layering:

- `_Channel` owns the Flight connection and the bearer header. It knows
  three wire operations: an action with a JSON (or text) body, a ticket read
  and a table upload.
- `ServerClient` is the typed surface. Every action is declared once in
  `_ACTION_DECODERS` with the function that turns its reply bytes into a
  Python value, so each public method is a payload plus one `_call`.
- `QueryRun` follows one submission by long-polling on the status revision
  (the server answers as soon as the revision moves past the one we hold,
  or after `wait_s`), and fetches its rows once it succeeded.
- `RemoteConnection` / `RemoteQuery` back `Session(endpoint=...)`.

The wire format (action names, JSON bodies, ticket shapes, status fields)
is the server's, crates/quail-server/src/lib.rs:188-475; the Python class
and method names are those of quail/remote/client.py.
"""

from __future__ import annotations

import json
import os
import time
from collections.abc import Callable, Iterator
from dataclasses import dataclass, fields

import pyarrow as pa
import pyarrow.flight as flight

TOKEN_VARIABLE = "QUAIL_SERVER_TOKEN"
TERMINAL_STATES = frozenset({"succeeded", "failed", "cancelled"})
POLL_S = 1.0


# --------------------------------------------------------------------------- status


@dataclass(frozen=True)
class QueryStatus:
    """One revision of a submission's status, as the server stored it."""

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
        """True once the submission can no longer change state."""
        return self.state in TERMINAL_STATES

    @classmethod
    def from_wire(cls, record: dict) -> "QueryStatus":
        # unknown keys from a newer server are dropped; lists become tuples so
        # the value stays hashable
        names = {f.name for f in fields(cls)}
        values = {}
        for key, val in record.items():
            if key in names:
                values[key] = tuple(val) if isinstance(val, list) and key in ("plans", "tables") else val
        return cls(**values)


class QueryFailedError(RuntimeError):
    """Raised when rows are asked of a submission that ended without any."""

    def __init__(self, status: QueryStatus):
        self.status = status
        why = status.error or "no error text was recorded"
        super().__init__(f"submission {status.id!r} ended as {status.state}: {why}")


# --------------------------------------------------------------------------- wire


class _Channel:
    """A Flight connection plus the call options every request carries."""

    def __init__(self, endpoint: str, token: str | None):
        self.endpoint = endpoint
        self.flight = flight.FlightClient(endpoint)
        if token is None:
            token = os.environ.get(TOKEN_VARIABLE)
        header = [(b"authorization", b"Bearer " + token.encode())] if token else []
        self.options = flight.FlightCallOptions(headers=header)

    def action(self, name: str, body) -> bytes:
        payload = body if isinstance(body, str) else json.dumps(body)
        replies = self.flight.do_action(flight.Action(name, payload.encode()), self.options)
        for reply in replies:       # every action answers with exactly one result
            return reply.body.to_pybytes()
        raise flight.FlightServerError(f"the server sent no reply to {name!r}")

    def read(self, ticket) -> flight.FlightStreamReader:
        raw = ticket if isinstance(ticket, str) else json.dumps(ticket)
        return self.flight.do_get(flight.Ticket(raw.encode()), self.options)

    def put(self, path: tuple, reader: pa.RecordBatchReader) -> None:
        descriptor = flight.FlightDescriptor.for_path(*path)
        writer, _ = self.flight.do_put(descriptor, reader.schema, self.options)
        with writer:
            for batch in reader:
                writer.write_batch(batch)

    def close(self) -> None:
        self.flight.close()


def _status(raw: bytes) -> QueryStatus:
    return QueryStatus.from_wire(json.loads(raw))


def _status_list(raw: bytes) -> list[QueryStatus]:
    return [QueryStatus.from_wire(r) for r in json.loads(raw)]


_ACTION_DECODERS: dict[str, Callable[[bytes], object]] = {
    "submit": _status,
    "status": _status,
    "cancel": _status,
    "list": _status_list,
    "answers": json.loads,
    "report": lambda raw: json.loads(raw)["regions"],
    "explain": lambda raw: raw.decode(),
}


def _as_reader(rows) -> pa.RecordBatchReader:
    if isinstance(rows, pa.RecordBatchReader):
        return rows
    return pa.RecordBatchReader.from_batches(rows.schema, rows.to_batches())


def _compact(**kw) -> dict:
    return {k: v for k, v in kw.items() if v is not None}


# --------------------------------------------------------------------------- client


class ServerClient:
    """Typed calls against one Quail Server."""

    def __init__(self, endpoint: str, token: str | None = None):
        self._channel = _Channel(endpoint, token)
        self.endpoint = endpoint

    def _call(self, action: str, payload=""):
        return _ACTION_DECODERS[action](self._channel.action(action, payload))

    def close(self) -> None:
        self._channel.close()

    # tables ------------------------------------------------------------
    def upload(self, name: str, table, id_col: str | None = None) -> None:
        """Make `table` (a Table or a RecordBatchReader) the server's table `name`."""
        path = (name,) if id_col is None else (name, id_col)
        self._channel.put(path, _as_reader(table))

    def sql(self, text: str) -> pa.Table:
        """Run `text` right away, outside the queue, and return its rows."""
        return self._channel.read(text).read_all()

    # the queue ---------------------------------------------------------
    def submit(self, sql: str, *, dialect: str | None = None, query_id: str | None = None,
               timeout_s: float | None = None) -> QueryStatus:
        return self._call("submit", _compact(sql=sql, dialect=dialect, id=query_id, timeout_s=timeout_s))

    def status(self, query_id: str, *, after: int | None = None, wait_s: float = 0.0) -> QueryStatus:
        """The current status; with `after`, wait up to `wait_s` for a revision past it."""
        if after is None:
            return self._call("status", query_id)
        return self._call("status", {"id": query_id, "after": after, "wait_s": wait_s})

    def cancel(self, query_id: str) -> QueryStatus:
        return self._call("cancel", query_id)

    def submissions(self) -> list[QueryStatus]:
        return self._call("list")

    def answers(self, query_id: str, *, after: int = 0, limit: int = 1000) -> dict:
        return self._call("answers", {"id": query_id, "after": after, "limit": limit})

    def report(self, query_id: str) -> list:
        return self._call("report", query_id)

    def explain(self, sql: str, dialect: str | None = None) -> str:
        return self._call("explain", _compact(sql=sql, dialect=dialect))

    def result_batches(self, query_id: str) -> pa.RecordBatchReader:
        """Rows saved by a submission that already succeeded."""
        return self._channel.read({"query_id": query_id}).to_reader()

    def stream_batches(self, query_id: str) -> pa.RecordBatchReader:
        """Rows of a submission; the server holds the stream open until it finishes."""
        return self._channel.read({"query_id": query_id, "stream": True}).to_reader()


class QueryRun:
    """Handle on one submission."""

    def __init__(self, client: ServerClient, query_id: str):
        self._client = client
        self.id = query_id

    def __repr__(self) -> str:
        return f"QueryRun(id={self.id!r})"

    def status(self) -> QueryStatus:
        return self._client.status(self.id)

    def watch(self, wait_s: float = POLL_S) -> Iterator[QueryStatus]:
        """Yield each new status revision, ending with the terminal one."""
        current = self.status()
        yield current
        while not current.done:
            nxt = self._client.status(self.id, after=current.revision, wait_s=wait_s)
            if nxt.revision != current.revision or nxt.done:
                yield nxt
            current = nxt

    def wait(self, wait_s: float = POLL_S, timeout_s: float | None = None) -> QueryStatus:
        """Block until the submission ends (or `timeout_s` passes) and return its status."""
        deadline = None if timeout_s is None else time.monotonic() + timeout_s
        last = None
        for last in self.watch(wait_s):
            if deadline is not None and time.monotonic() > deadline:
                break
        return last

    def cancel(self) -> QueryStatus:
        return self._client.cancel(self.id)

    def answers(self, after: int = 0, limit: int = 1000) -> dict:
        return self._client.answers(self.id, after=after, limit=limit)

    def report(self) -> list:
        return self._client.report(self.id)

    def _succeeded(self, wait_s: float) -> QueryStatus:
        final = self.wait(wait_s)
        if final.state != "succeeded":
            raise QueryFailedError(final)
        return final

    def stream_result(self, wait_s: float = POLL_S) -> pa.RecordBatchReader:
        self._succeeded(wait_s)
        return self._client.result_batches(self.id)

    def result(self, wait_s: float = POLL_S):
        from quail_b200.api.session import QueryResult
        final = self._succeeded(wait_s)
        rows = self._client.result_batches(self.id).read_all()
        plan_text = "\n".join(entry.get("text", "") for entry in final.plans)
        return QueryResult(table=rows, report={"regions": self.report()}, plan=plan_text)


# --------------------------------------------------------------------------- Session(endpoint=...)


class RemoteConnection:
    """What a remote Session holds: a client whose server owns the tables."""

    def __init__(self, endpoint: str, token: str | None = None):
        self.client = ServerClient(endpoint, token)

    def register(self, name: str, provider) -> None:
        from quail_b200.catalog.providers import ScanRequest, as_provider
        source = as_provider(provider)
        rows = source.scan(ScanRequest()) if hasattr(source, "scan") else source
        self.client.upload(name, rows, getattr(source, "id_col", None))

    def run(self, query_id: str) -> QueryRun:
        return QueryRun(self.client, query_id)

    def close(self) -> None:
        self.client.close()


def _rebatch(reader: pa.RecordBatchReader, batch_rows: int, limit: int | None) -> Iterator[pa.RecordBatch]:
    left = limit
    for batch in reader:
        if left is not None:
            if left <= 0:
                return
            batch = batch.slice(0, left)
            left -= batch.num_rows
        for start in range(0, batch.num_rows, batch_rows):
            yield batch.slice(start, batch_rows)


class RemoteQuery:
    """SQL text whose planning and execution happen on the server."""

    def __init__(self, session, text: str, dialect: str = "snowflake"):
        self.session = session
        self.text = text
        self.dialect = dialect

    @property
    def _client(self) -> ServerClient:
        return self.session._remote.client

    def submit(self, *, query_id: str | None = None, timeout_s: float | None = None) -> QueryRun:
        queued = self._client.submit(self.text, dialect=self.dialect, query_id=query_id, timeout_s=timeout_s)
        return QueryRun(self._client, queued.id)

    def run(self, plan=None, *, timeout_s: float | None = None):
        if plan is not None:
            raise ValueError("plans are made by the server; a remote query cannot take one")
        return self.submit(timeout_s=timeout_s).result()

    def collect(self, limit: int | None = None) -> pa.Table:
        rows = self.run().table
        return rows if limit is None else rows.slice(0, limit)

    def execute_stream(self, batch_rows: int = 65_536, limit: int | None = None, *,
                       timeout_s: float | None = None) -> pa.RecordBatchReader:
        if batch_rows < 1:
            raise ValueError(f"batch_rows={batch_rows}: at least one row per batch")
        if limit is not None and limit < 0:
            raise ValueError(f"limit={limit}: a row limit cannot be negative")
        source = self._client.stream_batches(self.submit(timeout_s=timeout_s).id)
        return pa.RecordBatchReader.from_batches(source.schema, _rebatch(source, batch_rows, limit))

    def explain(self, **_options) -> str:
        return self._client.explain(self.text, self.dialect)

    def plan(self):
        raise RuntimeError("the server plans remote queries; use explain() to read its plan")
