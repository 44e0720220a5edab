"""Data-parallel worker processes: one model replica per GPU.

The session's process spawns one worker per GPU (`CUDA_VISIBLE_DEVICES` =
that GPU), talks to each over a Unix socket with length-prefixed JSON frames,
and ships each region's documents as an Arrow IPC file in /dev/shm that the
worker maps (the C++ side is quail_b200._native: frames, spawn, shm).
Documents are hash-partitioned across the replicas by their content, so a
document and every question about it land on one GPU and each question is
asked once. Reference: crates/quail/src/workers.rs (spawn / connect / boot /
run_region / revive / interrupt, 120 s connect patience), stages.rs
(hash-partitioned stages) and shared.rs (/dev/shm tables).

Failure handling, host side only: a worker that exits or closes its socket
fails the region with its traceback; the next region revives (kills and
re-spawns) every worker, which reloads the model.

Copies larger than one GPU (`parallel="tp"` / `"ep"`, quail_b200.runtime.groups):
the workers of one copy see all of its GPUs and join one process group at
boot. tp: rows are sharded over copies and every rank of a copy gets its
copy's rows (rank 0's answers are kept); ep: every rank gets its own rows
and the ranks of a copy step in lockstep, so a rank with no rows still runs
(its experts serve the others).
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
import threading
import time
import zlib

import pyarrow as pa

from quail_b200 import _native

PATIENCE_MS = 120_000
MAX_FRAME = 1 << 34


class WorkerError(RuntimeError):
    pass


def _config_dict(config) -> dict:
    from dataclasses import asdict
    return asdict(config)


def docs_table(docs: list) -> pa.Table:
    if docs and not isinstance(docs[0], str) and docs[0] is not None and not isinstance(docs[0], (bytes,)):
        try:
            return pa.table({"doc": pa.array([list(map(int, d)) for d in docs], pa.list_(pa.int32()))})
        except TypeError:
            pass
    return pa.table({"doc": pa.array([None if d is None else str(d) for d in docs], pa.string())})


def table_bytes(t: pa.Table) -> bytes:
    sink = pa.BufferOutputStream()
    with pa.ipc.new_stream(sink, t.schema) as w:
        w.write_table(t)
    return sink.getvalue().to_pybytes()


def shard_of(doc, n: int) -> int:
    if isinstance(doc, str) or doc is None:
        b = ("" if doc is None else doc).encode()
    else:
        b = b",".join(str(int(x)).encode() for x in doc)
    return zlib.crc32(b) % n


class Worker:
    def __init__(self, index: int, pid: int, fd: int):
        self.index, self.pid, self.fd = index, pid, fd

    def call(self, msg: dict, timeout_ms: int = -1, on_event=None, on_ask=None) -> dict:
        """Send `msg` and return the reply; frames before it are events (to `on_event`)
        or asks (answered with on_ask(ask), by default "go on")."""
        _native.send_frame(self.fd, json.dumps(msg).encode(), timeout_ms)
        while True:
            reply = self.receive(timeout_ms)
            if "event" in reply:
                if on_event is not None:
                    on_event(self.index, reply["event"])
                continue
            if "ask" in reply:
                answer = on_ask(self.index, reply["ask"]) if on_ask is not None else {"stop": False}
                _native.send_frame(self.fd, json.dumps({"answer": answer}).encode(), timeout_ms)
                continue
            return reply

    def receive(self, timeout_ms: int = -1) -> dict:
        try:
            reply = json.loads(_native.recv_frame(self.fd, MAX_FRAME, timeout_ms))
        except _native.IpcClosed as exc:
            raise WorkerError(f"worker {self.index} closed its connection (exit status "
                              f"{_native.poll_exit(self.pid)})") from exc
        if "error" in reply:
            raise WorkerError(f"worker {self.index} failed:\n{reply['error']}")
        return reply


class WorkerPool:
    """`gpus` worker processes behind the session; same run_region as ModelEngine."""

    def __init__(self, config, python: str | None = None, boot: bool = True, registry=None):
        from quail_b200.api.config import check_config, group_size
        self.config = config
        self.cfg = check_config(config, registry)   # the decoder config (roles, prompt layout) the workers serve
        # a model only the session's registry knows travels to the workers as its config
        self._decoder = None if registry is None or registry.model(config.model) is None else self.cfg
        self.n = config.gpus
        # tp / ep: `group` workers form one model copy (rank = index % group)
        self.group = group_size(config)
        self.mode = config.parallel if self.group > 1 else "dp"
        self.copies = self.n // self.group
        self.python = python or sys.executable
        self.dir = tempfile.mkdtemp(prefix=f"qb-{os.getpid()}-")
        self.sock = os.path.join(self.dir, "s")
        self.listen_fd = _native.listen_unix(self.sock)
        self.workers: list[Worker] = []
        self._region = 0
        self.tokenizer = None
        self._interrupted = False
        self.ask_every_s = 0.25   # how often a worker asks whether to go on (regions with a stop hook)
        self._spawn()
        if boot:
            self.boot()

    # ------------------------------------------------------------ lifecycle
    def _spawn(self):
        pids = []
        ports = [_free_port() for _ in range(self.copies)] if self.group > 1 else []
        for i in range(self.n):
            env = [f"QB_WORKER_INDEX={i}"]
            if self.group > 1:
                copy, rank = divmod(i, self.group)
                gpus = ",".join(str(copy * self.group + k) for k in range(self.group))
                env += [f"CUDA_VISIBLE_DEVICES={gpus}", f"QB_GROUP_RANK={rank}", f"QB_GROUP_SIZE={self.group}",
                        f"QB_GROUP_PORT={ports[copy]}", "MASTER_ADDR=127.0.0.1"]
            elif self.config.device != "cpu":
                env.append(f"CUDA_VISIBLE_DEVICES={i}")
            argv = [self.python, "-m", "quail_b200.runtime.worker_main", "--socket", self.sock, "--index", str(i)]
            pids.append(_native.spawn(argv, env))
        fds = {}
        deadline = time.monotonic() + PATIENCE_MS / 1e3
        while len(fds) < self.n:
            for i, pid in enumerate(pids):
                st = _native.poll_exit(pid)
                if st >= 0 and i not in fds:
                    self._kill_all(pids)
                    raise WorkerError(f"worker {i} exited with status {st} before connecting")
            if time.monotonic() > deadline:
                self._kill_all(pids)
                raise WorkerError("workers did not connect within the patience")
            try:
                fd = _native.accept_unix(self.listen_fd, 200)
            except _native.IpcTimeout:
                continue
            hello = json.loads(_native.recv_frame(fd, 1 << 16, 10_000))
            fds[int(hello["index"])] = fd
        self.workers = [Worker(i, pids[i], fds[i]) for i in range(self.n)]

    @staticmethod
    def _kill_all(pids):
        for p in pids:
            _native.kill_pid(p, 9)
        for p in pids:
            for _ in range(100):
                if _native.poll_exit(p) != -1:
                    break
                time.sleep(0.01)

    def boot(self):
        msg = {"boot": _config_dict(self.config)}
        if self._decoder is not None:
            from dataclasses import asdict
            msg["decoder"] = asdict(self._decoder)
        replies = self._all(msg)
        self.boot_s = max(r.get("boot_s", 0.0) for r in replies)
        from quail_b200.api.tokenizer import load_tokenizer
        self.tokenizer = load_tokenizer(self.config.tokenizer or self.config.weights, self.cfg.vocab)

    def alive(self) -> bool:
        return all(_native.poll_exit(w.pid) == -1 for w in self.workers)

    def revive(self):
        """Kill and re-spawn every worker, then boot them again (models reload)."""
        self._kill_all([w.pid for w in self.workers])
        for w in self.workers:
            _native.close_fd(w.fd)
        self._spawn()
        self.boot()

    def interrupt(self):
        """Stop every worker now (the reference's Interrupter, workers.rs:687-711): running
        regions fail, and regions fail at once until resume()."""
        self._interrupted = True
        self._kill_all([w.pid for w in self.workers])

    def resume(self):
        """Accept regions again; the next one revives (re-spawns and boots) the workers."""
        self._interrupted = False

    def close(self):
        for w in self.workers:
            try:
                _native.send_frame(w.fd, json.dumps({"shutdown": True}).encode(), 2000)
            except _native.IpcError:
                pass
        t0 = time.monotonic()
        for w in self.workers:
            while _native.poll_exit(w.pid) == -1 and time.monotonic() - t0 < 10:
                time.sleep(0.02)
            if _native.poll_exit(w.pid) == -1:
                _native.kill_pid(w.pid, 9)
            _native.close_fd(w.fd)
        self.workers = []
        _native.close_fd(self.listen_fd)
        try:
            os.unlink(self.sock)
            os.rmdir(self.dir)
        except OSError:
            pass

    def _all(self, msg: dict, per_worker: list | None = None, on_event=None, on_ask=None) -> list:
        """Send to every worker (or per_worker messages), then gather every reply in order."""
        errors, replies = [], [None] * self.n

        def one(i):
            try:
                m = per_worker[i] if per_worker is not None else msg
                replies[i] = self.workers[i].call(m, on_event=on_event, on_ask=on_ask)
            except Exception as exc:  # noqa: BLE001 - every worker is told to finish; errors re-raised below
                errors.append(exc)

        threads = [threading.Thread(target=one, args=(i,)) for i in range(self.n)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return replies

    # ------------------------------------------------------------ regions
    def run_region(self, preamble: str, docs: list, calls: list, *, on_rows=None, stop=None):
        """Same contract as ModelEngine.run_region. on_rows(rows, values) receives each worker's
        finished rows while the region runs (session row numbers); stop() is asked by every
        worker about every `ask_every_s` and ends the region on all of them."""
        from dataclasses import asdict

        from quail_b200.api.engine import RegionOutput
        if self._interrupted:
            raise WorkerError("the session was interrupted; call resume() before the next query")
        if not self.alive():
            self.revive()
        self._region += 1
        shards = [[] for _ in range(self.n)]
        if self.mode == "tp":
            # rows go to copies; every rank of a copy runs its copy's rows
            for i, d in enumerate(docs):
                c = shard_of(d, self.copies)
                for r in range(self.group):
                    shards[c * self.group + r].append(i)
        else:
            for i, d in enumerate(docs):
                shards[shard_of(d, self.n)].append(i)
        from quail_b200.sql import guards as G
        paths, msgs = [], []
        for w in range(self.n):
            t = docs_table([docs[i] for i in shards[w]])
            name = f"qb-{os.getpid()}-{self._region}-{w}"
            path = _native.shm_write(name, table_bytes(t))
            paths.append(path)
            shard_calls = []
            for c in calls:
                d = asdict(c)
                d["guard"] = G.take(c.guard, shards[w])   # per-row guard inputs of this shard's rows
                shard_calls.append(d)
            region = {"preamble": preamble, "path": path, "calls": shard_calls}
            if on_rows is not None:
                region["events"] = True
            if stop is not None:
                region["ask_every_s"] = self.ask_every_s
            msgs.append({"region": region})

        def on_event(w, ev):
            if ev.get("kind") == "answers" and on_rows is not None:
                if self.mode == "tp" and w % self.group:
                    return
                for j, values in ev["rows"]:
                    on_rows([shards[w][j]], values)

        def on_ask(w, ask):
            return {"stop": bool(stop())} if stop is not None else {"stop": False}
        try:
            replies = self._all(None, msgs, on_event=on_event, on_ask=on_ask)
        finally:
            for p in paths:
                _native.unlink_path(p)
        from quail_b200.runtime.report import merge_worker_stats
        values = [None] * len(docs)
        counted = [not (self.mode == "tp" and w % self.group) for w in range(len(replies))]
        for w, rep in enumerate(replies):
            if not counted[w]:
                continue              # the other ranks of a tp copy computed the same answers
            for j, i in enumerate(shards[w]):
                values[i] = rep["values"][j]
        stats = merge_worker_stats([rep["stats"] for rep in replies], counted, len(docs))
        return RegionOutput(values=values, stats=stats)

    def run_pairs(self, preamble: str, anchors: list, pairs: list, call):
        """An AI join's pairs: each anchor (with all of its pairs) goes to one copy."""
        from dataclasses import asdict

        from quail_b200.api.engine import RegionOutput
        if not self.alive():
            self.revive()
        self._region += 1
        n_shards = self.copies if self.mode == "tp" else self.n
        owner = [shard_of(a, n_shards) for a in anchors]
        per = [[] for _ in range(n_shards)]
        for j, (i, _) in enumerate(pairs):
            per[owner[i]].append(j)
        paths, msgs = [], []
        for w in range(self.n):
            sh = w // self.group if self.mode == "tp" else w
            js = per[sh]
            local = {}
            for j in js:
                local.setdefault(pairs[j][0], len(local))
            a_tab = docs_table([anchors[i] for i in local] or [""])
            p_tab = pa.table({"anchor": pa.array([local[pairs[j][0]] for j in js], pa.int32()),
                              "doc": pa.array([pairs[j][1] for j in js], pa.string())})
            base = f"qb-{os.getpid()}-{self._region}-{w}"
            pa_path = _native.shm_write(base + "a", table_bytes(a_tab))
            pp_path = _native.shm_write(base + "p", table_bytes(p_tab))
            paths += [pa_path, pp_path]
            msgs.append({"pairs": {"preamble": preamble, "anchors": pa_path, "pairs": pp_path,
                                   "call": asdict(call)}})
        try:
            replies = self._all(None, msgs)
        finally:
            for p in paths:
                _native.unlink_path(p)
        from quail_b200.runtime.report import merge_worker_stats
        values = [None] * len(pairs)
        counted = [not (self.mode == "tp" and w % self.group) for w in range(len(replies))]
        for w, rep in enumerate(replies):
            if not counted[w]:
                continue
            sh = w // self.group if self.mode == "tp" else w
            for k, j in enumerate(per[sh]):
                values[j] = rep["values"][k]
        stats = merge_worker_stats([rep["stats"] for rep in replies], counted, len(pairs))
        return RegionOutput(values=values, stats=stats)

    @property
    def chunk_tokens(self):
        return self.config.chunk_tokens


def _free_port() -> int:
    """A TCP port on 127.0.0.1 that is free now (a tp / ep copy's rendezvous)."""
    import socket
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def content_hash(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()[:16]
