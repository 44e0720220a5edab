"""Quail Server: a session behind Arrow Flight, with a persistent query queue.

Calls (the reference's surface, crates/quail-server/src/lib.rs:188-475):

  DoPut     descriptor path [name] or [name, id column]: register the
            uploaded rows as a table of the server's session.
  DoGet     ticket {"query_id": id}: the saved rows of a submission that
            succeeded; {"query_id": id, "stream": true}: its rows once it
            finishes (waiting while it is queued or running; an error if it
            failed or was cancelled); any other ticket is SQL, run at once.
  DoAction  explain {sql, dialect} -> plan text; submit {sql, dialect, id,
            timeout_s} -> status; status id | {id, after, wait_s} -> status;
            answers {id, after, limit} -> {answers, next}; report id ->
            {regions}; cancel id -> status; list -> [status].

With QUAIL_SERVER_TOKEN set (or `token=`), every call must carry the header
`authorization: Bearer <token>`; others are refused as unauthenticated.
The transport is Arrow's C++ Flight (gRPC) through pyarrow.flight.
"""

from __future__ import annotations

import json
import os

import pyarrow as pa
import pyarrow.flight as flight

from quail_b200.server.queue import SubmissionQueue

TOKEN_VARIABLE = "QUAIL_SERVER_TOKEN"

ACTIONS = [
    ("explain", "Return a query's plan: {sql, dialect}"),
    ("submit", "Queue a query: {sql, dialect, id, timeout_s}"),
    ("status", "Return a submission's status: id, or {id, after, wait_s}"),
    ("answers", "Return a run's answer events: {id, after, limit}"),
    ("report", "Return each model region's report of a submission that succeeded, by id"),
    ("cancel", "Stop a submission, by id"),
    ("list", "Return every submission"),
]


class _TokenMiddlewareFactory(flight.ServerMiddlewareFactory):
    def __init__(self, token: str):
        self.expected = f"Bearer {token}"

    def start_call(self, info, headers):
        got = headers.get("authorization") or headers.get("Authorization") or []
        if self.expected not in got:
            raise flight.FlightUnauthenticatedError("a bearer token is required")
        return None


def _json(value) -> bytes:
    return json.dumps(value, default=str).encode()


class QuailFlightServer(flight.FlightServerBase):
    def __init__(self, session, data_dir: str, location: str = "grpc://127.0.0.1:0", token: str | None = None):
        token = token if token is not None else os.environ.get(TOKEN_VARIABLE) or None
        mw = {"auth": _TokenMiddlewareFactory(token)} if token else None
        super().__init__(location, middleware=mw)
        self.session = session
        self.queue = SubmissionQueue(data_dir, session)
        self._uploads = 0

    @property
    def endpoint(self) -> str:
        return f"grpc://127.0.0.1:{self.port}"

    # ------------------------------------------------------------ DoPut
    def do_put(self, context, descriptor, reader, writer):
        path = [p.decode() if isinstance(p, bytes) else p for p in (descriptor.path or [])]
        if not path:
            raise flight.FlightServerError("an upload's descriptor path names its table")
        name, id_col = path[0], (path[1] if len(path) > 1 else None)
        table = reader.read_all()
        if id_col is not None and id_col not in table.column_names:
            raise flight.FlightServerError(f"the table has no id column {id_col}")
        from quail_b200.catalog.providers import DocumentProvider
        self.session.register(name, DocumentProvider.from_table(table, id_col=id_col) if id_col else table)
        self._uploads += 1

    # ------------------------------------------------------------ DoGet
    def do_get(self, context, ticket):
        text = ticket.ticket.decode()
        try:
            asked = json.loads(text)
        except ValueError:
            asked = None
        if isinstance(asked, dict) and "query_id" in asked:
            sid = asked["query_id"]
            if asked.get("stream"):
                st = self.queue.wait_finished(sid)
                if st["state"] != "succeeded":
                    raise flight.FlightServerError(f"query {sid} {st['state']}: {st.get('error')}")
            try:
                table = self.queue.rows(sid)
            except KeyError as exc:
                raise flight.FlightServerError(str(exc)) from None
            return flight.RecordBatchStream(table)
        table = self.session.sql(text).collect()
        return flight.RecordBatchStream(table)

    # ------------------------------------------------------------ DoAction
    def list_actions(self, context):
        return ACTIONS

    def do_action(self, context, action):
        body = action.body.to_pybytes().decode() if action.body is not None else ""
        kind = action.type
        q = self.queue
        try:
            if kind == "explain":
                asked = json.loads(body) if body.startswith("{") else {"sql": body}
                out = self.session.sql(asked["sql"], asked.get("dialect") or "snowflake").explain().encode()
            elif kind == "submit":
                asked = json.loads(body)
                out = _json(q.submit(asked["sql"], asked.get("dialect"), asked.get("id"), asked.get("timeout_s")))
            elif kind == "status":
                if body.startswith("{"):
                    asked = json.loads(body)
                    st = q.status_after(asked["id"], int(asked.get("after", 0)), float(asked.get("wait_s", 0.0)))
                else:
                    st = q.status(body)
                if st is None:
                    raise KeyError(f"no submission {body!r}")
                out = _json(st)
            elif kind == "answers":
                asked = json.loads(body)
                out = _json(q.answers_of(asked["id"], int(asked.get("after", 0)), int(asked.get("limit", 1000))))
            elif kind == "report":
                out = _json({"regions": q.report(body)})
            elif kind == "cancel":
                out = _json(q.cancel(body))
            elif kind == "list":
                out = _json(q.list())
            else:
                raise flight.FlightServerError(f"unknown action {kind!r}")
        except KeyError as exc:
            raise flight.FlightServerError(f"not found: {exc}") from None
        except (ValueError, TypeError) as exc:
            raise flight.FlightServerError(f"invalid request: {exc}") from None
        return [flight.Result(pa.py_buffer(out))]

    def shutdown(self):
        self.queue.close()
        super().shutdown()


def serve(session, data_dir: str, host: str = "127.0.0.1", port: int = 0, token: str | None = None,
          block: bool = True) -> QuailFlightServer:
    """Start a server on `host:port` (0: any free port). With block, serve until interrupted."""
    server = QuailFlightServer(session, data_dir, f"grpc://{host}:{port}", token=token)
    if block:
        try:
            server.serve()
        except KeyboardInterrupt:
            pass
        finally:
            server.shutdown()
    return server
