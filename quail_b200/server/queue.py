"""The server's submitted queries: run one at a time, kept on disk.

Every submission has a directory under the server's data directory:

  status.json    the status (id, sql, dialect, state, error, timeout_s,
                 submitted/started/finished times, num_rows, revision, plans,
                 ready, num_answers, tables), rewritten atomically (write a
                 new file, then rename) at every change
  result.arrow   the rows, once the query succeeded (Arrow IPC file)
  report.json    each model region's report, once it succeeded
  answers.json   the run's answer events

A server opened on a directory an earlier server used lists its
submissions; one that was queued or running when that server stopped is
marked failed ("the server stopped before the query finished"). Submitting
an id that exists returns its status and runs nothing. A status reader can
wait for the next revision (`status_after`). Cancelling a queued submission
removes it from the queue; cancelling the running one stops its executor
between two forward passes. A submission with `timeout_s` is stopped the
same way once it has run that long.

Reference behavior: crates/quail-server/src/queue.rs (Queue::open, submit,
status_after, answers, report, cancel, rows, run; `save` at :639-646).
"""

from __future__ import annotations

import json
import os
import threading
import time
import uuid
from collections import deque

import pyarrow as pa
import pyarrow.ipc as ipc

STOPPED = "the server stopped before the query finished"
FINISHED = ("succeeded", "failed", "cancelled")


def _now() -> float:
    return time.time()


class SubmissionQueue:
    """Submissions by id, a FIFO of waiting ids, and one runner thread."""

    def __init__(self, directory: str, session):
        self.directory = directory
        self.session = session
        os.makedirs(directory, exist_ok=True)
        self._lock = threading.Lock()
        self._changed = threading.Condition(self._lock)
        self.subs: dict[str, dict] = {}
        self.waiting: deque[str] = deque()
        self.running: str | None = None
        self._stop_reason: str | None = None
        self._interrupt = threading.Event()
        self.answers: dict[str, list] = {}
        self.closed = False
        for name in sorted(os.listdir(directory)):
            path = os.path.join(directory, name, "status.json")
            if not os.path.exists(path):
                continue
            with open(path) as f:
                st = json.load(f)
            if st.get("state") not in FINISHED:
                st.update(state="failed", error=STOPPED, finished_at=_now(), revision=st.get("revision", 0) + 1)
                self._save(st)
            self.subs[st["id"]] = st
        self._runner = threading.Thread(target=self._run, name="quail-queue", daemon=True)
        self._runner.start()

    # ------------------------------------------------------------ persistence
    def _home(self, sid: str) -> str:
        return os.path.join(self.directory, sid)

    def _save(self, st: dict) -> None:
        home = self._home(st["id"])
        os.makedirs(home, exist_ok=True)
        tmp = os.path.join(home, "status.json.new")
        with open(tmp, "w") as f:
            json.dump(st, f)
        os.replace(tmp, os.path.join(home, "status.json"))

    def _update(self, sid: str, **changes) -> dict:
        """Change a status under the lock, bump its revision, save it, wake the waiters."""
        st = self.subs[sid]
        st.update(changes)
        st["revision"] = st.get("revision", 0) + 1
        self._save(st)
        self._changed.notify_all()
        return dict(st)

    # ------------------------------------------------------------ calls
    def submit(self, sql: str, dialect: str | None = None, sid: str | None = None,
               timeout_s: float | None = None) -> dict:
        with self._lock:
            if self.closed:
                raise RuntimeError("the server is stopping")
            if sid is not None and sid in self.subs:
                return dict(self.subs[sid])
            sid = sid or uuid.uuid4().hex[:16]
            if "/" in sid or sid.startswith("."):
                raise ValueError(f"invalid submission id {sid!r}")
            st = {"id": sid, "sql": sql, "dialect": dialect, "state": "queued", "error": None,
                  "timeout_s": timeout_s, "submitted_at": _now(), "started_at": None, "finished_at": None,
                  "num_rows": None, "revision": 0, "plans": [], "ready": False, "num_answers": 0, "tables": []}
            self.subs[sid] = st
            self.waiting.append(sid)
            return self._update(sid)

    def status(self, sid: str) -> dict | None:
        with self._lock:
            st = self.subs.get(sid)
            return dict(st) if st is not None else None

    def status_after(self, sid: str, after: int, wait_s: float) -> dict | None:
        """The status once its revision is above `after`, or after `wait_s` seconds (60 at most)."""
        deadline = time.monotonic() + max(0.0, min(float(wait_s), 60.0))
        with self._lock:
            while True:
                st = self.subs.get(sid)
                if st is None:
                    return None
                if st.get("revision", 0) > after:
                    return dict(st)
                left = deadline - time.monotonic()
                if left <= 0:
                    return dict(st)
                self._changed.wait(left)

    def list(self) -> list[dict]:
        with self._lock:
            return [dict(s) for s in sorted(self.subs.values(), key=lambda s: s["submitted_at"])]

    def cancel(self, sid: str) -> dict:
        with self._lock:
            st = self.subs.get(sid)
            if st is None:
                raise KeyError(f"no submission {sid!r}")
            if st["state"] == "queued":
                self.waiting.remove(sid)
                return self._update(sid, state="cancelled", error="cancelled", finished_at=_now())
            if st["state"] == "running":
                self._stop_reason = "cancelled"
                self._interrupt.set()
            return dict(st)

    def answers_of(self, sid: str, after: int = 0, limit: int = 1000) -> dict:
        with self._lock:
            if sid not in self.subs:
                raise KeyError(f"no submission {sid!r}")
            events = self.answers.get(sid)
        if events is None:
            path = os.path.join(self._home(sid), "answers.json")
            events = json.load(open(path)) if os.path.exists(path) else []
        start = min(max(after, 0), len(events))
        end = min(start + max(limit, 0), len(events))
        return {"answers": events[start:end], "next": end}

    def report(self, sid: str) -> list:
        self._succeeded(sid)
        with open(os.path.join(self._home(sid), "report.json")) as f:
            return json.load(f)

    def rows(self, sid: str) -> pa.Table:
        self._succeeded(sid)
        with pa.memory_map(os.path.join(self._home(sid), "result.arrow")) as src:
            return ipc.open_file(src).read_all()

    def wait_finished(self, sid: str, timeout: float | None = None) -> dict:
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._lock:
            while True:
                st = self.subs.get(sid)
                if st is None:
                    raise KeyError(f"no submission {sid!r}")
                if st["state"] in FINISHED:
                    return dict(st)
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    return dict(st)
                self._changed.wait(left if left is not None else 1.0)

    def _succeeded(self, sid: str) -> None:
        st = self.status(sid)
        if st is None:
            raise KeyError(f"no submission {sid!r}")
        if st["state"] != "succeeded":
            raise KeyError(f"submission {sid!r} is {st['state']}, not succeeded")

    def close(self) -> None:
        with self._lock:
            self.closed = True
            self._stop_reason = STOPPED
            self._interrupt.set()
            self._changed.notify_all()
        self._runner.join(timeout=30)

    # ------------------------------------------------------------ runner
    def _run(self) -> None:
        while True:
            with self._lock:
                while not self.waiting and not self.closed:
                    self._changed.wait(1.0)
                if self.closed:
                    return
                sid = self.waiting.popleft()
                self.running = sid
                self._stop_reason = None
                self._interrupt.clear()
                st = self._update(sid, state="running", started_at=_now())
            timer = None
            if st.get("timeout_s"):
                def expire():
                    with self._lock:
                        if self.running == sid and self._stop_reason is None:
                            self._stop_reason = f"timed out after {st['timeout_s']} s"
                            self._interrupt.set()
                timer = threading.Timer(float(st["timeout_s"]), expire)
                timer.daemon = True
                timer.start()
            try:
                table, report, plan_text = self._execute(sid, st["sql"], st.get("dialect"))
                home = self._home(sid)
                with ipc.new_file(os.path.join(home, "result.arrow"), table.schema) as w:
                    w.write_table(table)
                with open(os.path.join(home, "report.json"), "w") as f:
                    json.dump([report], f, default=str)
                events = self.answers.get(sid, [])
                with open(os.path.join(home, "answers.json"), "w") as f:
                    json.dump(events, f, default=str)
                with self._lock:
                    self._update(sid, state="succeeded", finished_at=_now(), num_rows=table.num_rows,
                                 plans=[{"text": plan_text, "estimated_seconds": report.get("estimated_s", 0.0)}],
                                 num_answers=len(events))
            except Exception as exc:  # noqa: BLE001 - every failure is recorded in the status
                with self._lock:
                    reason = self._stop_reason
                    state = "cancelled" if reason == "cancelled" else "failed"
                    self._update(sid, state=state, finished_at=_now(), error=reason or f"{type(exc).__name__}: {exc}")
            finally:
                if timer is not None:
                    timer.cancel()
                with self._lock:
                    self.running = None

    def _execute(self, sid: str, sql: str, dialect: str | None):
        """Run one query on the session; the engine's executor checks the interrupt between passes."""
        q = self.session.sql(sql, dialect or "snowflake")
        engine = self.session.engine() if self.session._needs_model(q.tree) else None
        if engine is not None:
            engine.interrupt = self._interrupt
            with self._lock:
                self._update(sid, ready=True)
        if self._interrupt.is_set():
            raise RuntimeError("stopped before the run started")
        result = q.run()
        if self._interrupt.is_set():
            raise RuntimeError(self._stop_reason or "stopped")
        events = [{"region": 0, "kind": "rows", "rows": result.table.num_rows,
                   "evaluated_documents": result.report.get("evaluated_documents", 0)}]
        self.answers[sid] = events
        return result.table, dict(result.report), result.plan
