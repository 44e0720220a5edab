"""A worker process: loads one model replica and serves regions over its socket.

    python -m quail_b200.runtime.worker_main --socket PATH --index I

Messages (JSON frames): {"boot": config} -> {"ready": true, "boot_s": s};
{"region": {"preamble", "path", "calls"}} -> {"values": [...], "stats": {...}};
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
                cfg = dict(msg["boot"])
                cfg["gpus"] = 1
                t0 = time.perf_counter()
                from quail_b200.api.engine import ModelEngine
                engine = ModelEngine(EngineConfig(**cfg))
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
                out = engine.run_region(r["preamble"], docs, calls) if docs else None
                reply = {"values": out.values if out else [], "stats": out.stats if out else {}}
                del table, mapped
            else:
                reply = {"error": f"unknown message {sorted(msg)}"}
        except Exception:  # noqa: BLE001 - the traceback goes back to the session
            reply = {"error": traceback.format_exc()}
        _native.send_frame(fd, json.dumps(reply).encode(), -1)


if __name__ == "__main__":
    main()
