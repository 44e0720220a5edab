"""A worker process: loads one model replica and serves regions over its socket.

    python -m quail_b200.runtime.worker_main --socket PATH --index I

Messages (JSON frames): {"boot": config} -> {"ready": true, "boot_s": s};
{"region": {"preamble", "path", "calls"}} -> {"values": [...], "stats": {...}};
{"pairs": {"preamble", "anchors", "pairs", "call"}} (an AI join's pairs) -> the same;
during a region the worker may also send {"event": ...} frames and {"ask": ...}
frames that the session answers (`_Channel`);
{"shutdown": true} -> exit. A failure answers {"error": traceback} and the
worker keeps serving (the reference's WorkerEnd.fail, worker.py:410).
"""

from __future__ import annotations

import argparse
import json
import time
import traceback


def _inject_fault(index: int) -> None:
    """Host-side fault injection for the runtime tests (no GPU is involved).

    QB_FAULT=raise:<index> makes that worker fail its regions with an
    exception; QB_FAULT=exit:<index> makes it exit in the middle of a region.
    """
    import os
    spec = os.environ.get("QB_FAULT", "")
    if ":" not in spec:
        return
    kind, who = spec.split(":", 1)
    if int(who) != index:
        return
    if kind == "raise":
        raise RuntimeError(f"injected failure in worker {index}")
    if kind == "exit":
        os._exit(3)


class _Channel:
    """The worker's side of a region's ask channel (the reference's Connection::call,
    crates/quail/src/workers.rs:184-213).

    While a region runs, the worker may send frames before its reply:
    {"event": {"kind": "answers", "rows": [[row, values], ...]}} with the rows
    whose questions are all answered, and {"event": {"kind": "progress", ...}};
    neither expects an answer. With `ask_every_s`, it also asks
    {"ask": {"kind": "continue", "done": n}} at most that often, between forward
    passes, and waits for {"answer": {"stop": bool}}: a host whose LIMIT is
    met, or whose query was cancelled, answers stop and the region ends with
    the rows finished so far.
    """

    def __init__(self, fd, events: bool, ask_every_s):
        self.fd = fd
        self.events = bool(events)
        self.asks = ask_every_s is not None
        self.every = float(ask_every_s or 0.0)
        self.rows: list = []
        self.done = 0
        self.last = time.monotonic()

    def _send(self, obj) -> None:
        from quail_b200 import _native
        _native.send_frame(self.fd, json.dumps(obj).encode(), -1)

    def on_rows(self, rows, values) -> None:
        for i in rows:
            self.rows.append([i, values])
        self.done += len(rows)
        if len(self.rows) >= 64 or time.monotonic() - self.last > 0.2:
            self.flush()

    def flush(self) -> None:
        if self.events and self.rows:
            self._send({"event": {"kind": "answers", "rows": self.rows}})
            self._send({"event": {"kind": "progress", "rows_done": self.done}})
            self.rows = []
        self.last = time.monotonic()

    def should_stop(self) -> bool:
        from quail_b200 import _native
        if time.monotonic() - self.last < self.every:
            return False
        self.flush()
        self._send({"ask": {"kind": "continue", "done": self.done}})
        reply = json.loads(_native.recv_frame(self.fd, 1 << 20, 120_000))
        return bool(reply.get("answer", {}).get("stop", False))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--socket", required=True)
    ap.add_argument("--index", type=int, required=True)
    args = ap.parse_args()
    from quail_b200.utils.progress import set_gpu_index
    set_gpu_index(args.index)
    from quail_b200 import _native
    import os
    if os.environ.get("QB_FAULT") == f"noconnect:{args.index}":
        raise SystemExit(4)
    fd = _native.connect_unix(args.socket, 120_000)
    _native.send_frame(fd, json.dumps({"index": args.index}).encode(), 10_000)
    engine = None
    while True:
        try:
            msg = json.loads(_native.recv_frame(fd, 1 << 30, -1))
        except _native.IpcClosed:
            return
        try:
            if "shutdown" in msg:
                if engine is not None:
                    engine.close()
                return
            if "boot" in msg:
                from quail_b200.api.config import EngineConfig
                from quail_b200.runtime.groups import build_group_engine, group_env
                cfg = dict(msg["boot"])
                t0 = time.perf_counter()
                registry = None
                if "decoder" in msg:
                    # a model the session's extension registry added
                    from quail_b200.extensions import built_in_registry
                    from quail_b200.models.config import DecoderConfig
                    registry = built_in_registry()
                    d = dict(msg["decoder"])
                    d["layer_kinds"] = tuple(d.get("layer_kinds") or ())
                    registry.register_model(cfg["model"], DecoderConfig(**d))
                grp = group_env()
                if grp is not None:
                    engine = build_group_engine(EngineConfig(**cfg), *grp)
                else:
                    from quail_b200.api.engine import ModelEngine
                    cfg["gpus"] = 1
                    engine = ModelEngine(EngineConfig(**cfg), registry=registry)
                reply = {"ready": True, "boot_s": time.perf_counter() - t0}
            elif "region" in msg:
                import pyarrow as pa
                _inject_fault(args.index)

                from quail_b200.api.engine import CallSpec
                r = msg["region"]
                mapped = _native.MappedFile(r["path"])
                table = pa.ipc.open_stream(pa.py_buffer(memoryview(mapped))).read_all()
                docs = table.column("doc").to_pylist()
                calls = [CallSpec(**c) for c in r["calls"]]
                # a rank of a multi-GPU copy runs even with no rows: its peers wait for its passes
                grouped = getattr(engine, "group", None) is not None
                chan = _Channel(fd, r.get("events", False), r.get("ask_every_s"))
                out = (engine.run_region(r["preamble"], docs, calls, on_rows=chan.on_rows if chan.events else None,
                                         stop=chan.should_stop if chan.asks else None)
                       if docs or grouped else None)
                chan.flush()
                reply = {"values": out.values if out else [], "stats": out.stats if out else {}}
                del table, mapped
            elif "pairs" in msg:
                import pyarrow as pa

                from quail_b200.api.engine import CallSpec
                r = msg["pairs"]
                tabs = []
                for key in ("anchors", "pairs"):
                    mapped = _native.MappedFile(r[key])
                    tabs.append(pa.ipc.open_stream(pa.py_buffer(memoryview(mapped))).read_all())
                    del mapped
                anchors = tabs[0].column("doc").to_pylist()
                pairs = list(zip(tabs[1].column("anchor").to_pylist(), tabs[1].column("doc").to_pylist()))
                grouped = getattr(engine, "group", None) is not None
                if pairs or grouped:
                    out = engine.run_pairs(r["preamble"], anchors, pairs, CallSpec(**r["call"]))
                    reply = {"values": out.values, "stats": out.stats}
                else:
                    reply = {"values": [], "stats": {}}
            else:
                reply = {"error": f"unknown message {sorted(msg)}"}
        except Exception:  # noqa: BLE001 - the traceback goes back to the session
            reply = {"error": traceback.format_exc()}
        _native.send_frame(fd, json.dumps(reply).encode(), -1)


if __name__ == "__main__":
    main()
