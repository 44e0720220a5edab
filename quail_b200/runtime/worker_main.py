"""A worker process: loads one model replica and serves regions over its socket.

    python -m quail_b200.runtime.worker_main --socket PATH --index I

Messages (JSON frames): {"boot": config} -> {"ready": true, "boot_s": s};
{"region": {"preamble", "path", "calls"}} -> {"values": [...], "stats": {...}};
{"pairs": {"preamble", "anchors", "pairs", "call"}} (an AI join's pairs) -> the same;
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
                from quail_b200.runtime.groups import build_group_engine, group_env
                cfg = dict(msg["boot"])
                t0 = time.perf_counter()
                grp = group_env()
                if grp is not None:
                    engine = build_group_engine(EngineConfig(**cfg), *grp)
                else:
                    from quail_b200.api.engine import ModelEngine
                    cfg["gpus"] = 1
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
                # a rank of a multi-GPU copy runs even with no rows: its peers wait for its passes
                grouped = getattr(engine, "group", None) is not None
                out = engine.run_region(r["preamble"], docs, calls) if docs or grouped else None
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
