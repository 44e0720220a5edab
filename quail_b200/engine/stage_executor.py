"""The per-GPU prefill scheduler: admission, chunk packing, forward, readout.

Work arrives as `Task`s: a sequence of new tokens that writes one arena key
and reads earlier keys (the shared instruction prefix, a document another
task wrote). The executor packs the tasks at the head of the queue into a
chunk of at most `chunk_tokens` new tokens, splitting a task that does not
fit into prefill pieces (chunked prefill over its own pages), and admits a
task only when

  - every key it reads was fully written by an already launched chunk
    (stream order then guarantees the KV is there), and
  - its own pages fit in the free pool (after evicting retained keys).

While the GPU runs chunk k the host packs and launches chunk k+1, then
collects chunk k's readout (one pinned D2H copy + an event) and hands each
readout row to its task's `on_done`, which may submit follow-up tasks (a
CLASSIFY on the rows an AI.IF kept reads the same document pages).

Reference behavior: quail/backends/quail/executor/stage_executor.py
(StageExecutor.run, _run_one, forward_chunk), admission.py (next_chunk,
prefill pieces, Borrowing) and readout.py (async readouts drained in order).
"""

from __future__ import annotations

import os

import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable

import numpy as np
import torch

from quail_b200.engine.arena import ArenaFullError
from quail_b200.engine.chunk import ChunkPacker, SeqSpec


class OversizedDocumentError(ArenaFullError):
    """A single task needs more pages than the whole arena has."""


class QueryCancelled(RuntimeError):
    """The executor's stop hook asked it to stop between passes."""


@dataclass
class Task:
    key: object
    tokens: np.ndarray
    pos_start: int
    reads: list = field(default_factory=list)       # [(key, tokens)]
    readout: bool = False
    on_done: Callable | None = None                  # on_done(task, logits_row | None)
    free_after: bool = True
    own_prefix: int = 0                              # own tokens already resident (continuation)
    done: int = 0                                    # new tokens already launched
    tag: object = None
    readout_rows: tuple | None = None                # offsets read out (default: the last token)
    full_readout: bool = False                       # also argmax / log-sum-exp over the vocabulary
    topk: bool = False                               # and the top-k token ids and logits
    reserve_tokens: int = 0                          # decode headroom allocated with the key's pages
    got_rows: list = field(default_factory=list)     # readout rows of the pieces already collected
    np_rows: bool = False                            # on_done gets numpy rows (views of the pass's host copy)
    # a document-isolated block: its own tokens read each other both ways, so it runs in one
    # pass (never split into prefill pieces)
    bidirectional: bool = False

    @property
    def remaining(self) -> int:
        return len(self.tokens) - self.done


@dataclass
class _Replayed:
    """What the executor keeps of a pass that ran as a graph replay."""

    num_tokens: int
    upload_bytes: int


@dataclass
class ExecutorStats:
    passes: int = 0
    tokens: int = 0
    readouts: int = 0
    gpu_ms: float = 0.0
    pass_tokens: list = field(default_factory=list)
    pass_rows: list = field(default_factory=list)
    h2d_bytes: int = 0
    d2h_bytes: int = 0
    wall_s: float = 0.0
    evictions: int = 0          # retained keys freed to make room
    reused: int = 0             # documents a region found retained (no prefill)
    replays: int = 0            # documents a region recomputed because their retained KV was evicted
    cached: int = 0             # prompt tokens tasks read from resident KV instead of computing them
    tree_passes: int = 0        # passes whose attention ran the tree path (stacked shared segments)


ANSWER_ADMISSION_ENV = "QUAIL_ANSWER_ADMISSION"
ANSWER_ADMISSION_MODES = ("headroom=0", "headroom")
HEADROOM_TRACE_ENV = "QUAIL_HEADROOM_TRACE"


def answer_admission_mode() -> str:
    """How a task's decode headroom counts at admission (the reference's QUAIL_ANSWER_ADMISSION,
    quail/backends/quail/executor/stage_executor.py:27-50): "headroom" (default) admits a
    task when its prompt and its answer's headroom fit; "headroom=0" when its prompt fits
    (a decode step then grows the key's pages, evicting retained KV if it must)."""
    mode = os.environ.get(ANSWER_ADMISSION_ENV, "headroom")
    if mode not in ANSWER_ADMISSION_MODES:
        raise ValueError(f"{ANSWER_ADMISSION_ENV}={mode!r}; expected one of {', '.join(ANSWER_ADMISSION_MODES)}")
    return mode


class StageExecutor:
    def __init__(self, model, arena, chunk_tokens: int, *, min_piece: int = 64, gpu_timing: bool = False,
                 max_seqs: int | None = None, cont_cap: int = 512, attention: str = "unified"):
        self.model = model
        self.arena = arena
        self.pool = arena.pool
        self.chunk_tokens = chunk_tokens
        self.min_piece = min_piece
        self.max_seqs = max_seqs
        # continuations (decode steps) per pass: with more decoding rows than this they
        # split into groups that alternate, so the host builds one group's next step
        # while the GPU runs the other's (a step depends on the previous one's token)
        self.cont_cap = cont_cap
        self.device = arena.device
        # the attention path: "unified", "tree" (stack readers of a shared first segment) or "auto"
        self.packer = ChunkPacker(self.pool, self.device, tree=attention)
        self.queue: deque[Task] = deque()
        # continuations of resident keys (decode steps, label continuations):
        # admitted before new work, they need at most a page-list extension
        self.cont: deque[Task] = deque()
        self.follow: deque[Task] = deque()   # new keys that read a resident document (follow-up questions)
        self.written: dict = {}     # key -> tokens written by launched chunks
        self.stats = ExecutorStats()
        self.gpu_timing = gpu_timing and self.device.type == "cuda"
        self.graphs = None        # engine.graphs.DecodeGraphs once enable_graphs() is called
        # QB_NVTX=1: one NVTX range per forward pass (named by pass index and sequence count)
        self.nvtx = self.device.type == "cuda" and os.environ.get("QB_NVTX") == "1"
        self._inflight: deque = deque()
        self.should_stop: Callable | None = None   # checked between passes (cancel / timeout)
        self.answer_headroom = answer_admission_mode() == "headroom"
        # QUAIL_HEADROOM_TRACE=<dir>: each run writes its arena occupancy per pass there
        # (seconds since the run began, pass, new tokens, free / held pages, keys held, retained
        # keys, and the device memory allocated when the pass launched)
        self.trace_dir = os.environ.get(HEADROOM_TRACE_ENV) or None
        self.trace: list = []

    # ------------------------------------------------------------ submission
    def submit(self, task: Task) -> None:
        need = self.pool.pages_needed(task.own_prefix + len(task.tokens))
        if need > self.pool.num_pages:
            raise OversizedDocumentError(
                f"task {task.key!r} needs {need} pages; the arena has {self.pool.num_pages}")
        if task.own_prefix > 0 and self.pool.resident(task.key):
            self.cont.append(task)
        elif len(task.reads) > 1:
            self.follow.append(task)   # reads a document as well as the prefix: a follow-up
        else:
            self.queue.append(task)

    def submit_continuation(self, task: Task) -> None:
        """A continuation of a resident key (a decode step): straight to the continuation queue."""
        self.cont.append(task)

    def free(self, key) -> None:
        self.pool.free_key(key)
        self.written.pop(key, None)

    def rewind(self, key, tokens: int) -> None:
        """Trim a key to its first `tokens` tokens (KV rewind: a decode's own tokens dropped once
        no one reads them), releasing the pages past them."""
        self.pool.rewind(key, tokens)
        if key in self.written:
            self.written[key] = min(self.written[key], tokens)

    def retain(self, key, as_key) -> None:
        """Keep a finished key's KV under `as_key` for a later region; it is evicted (freed) first
        when the arena runs short, and a region that needs it then recomputes it."""
        if self.pool.resident(as_key):
            self.free(as_key)          # an older copy of the same document's KV
        self.pool.adopt(key, as_key)
        self.written[as_key] = self.written.pop(key, self.pool.tokens[as_key])
        self.pool.retain(as_key)

    def claim(self, retained_key, key) -> bool:
        """Take a retained key's KV for `key` (pinned again: not evictable); False if it was evicted."""
        if not self.pool.resident(retained_key):
            self.written.pop(retained_key, None)
            return False
        self.pool.adopt(retained_key, key)
        self.written[key] = self.written.pop(retained_key, self.pool.tokens[key])
        return True

    def _evict(self, pages: int) -> None:
        for key in self.pool.evict_retained(pages):
            self.written.pop(key, None)
            self.stats.evictions += 1

    # ------------------------------------------------------------ admission
    def _readable(self, task: Task) -> bool:
        return all(self.written.get(k, -1) >= n for k, n in task.reads)

    def _admit(self) -> list[SeqSpec]:
        room = self.chunk_tokens
        specs: list[SeqSpec] = []
        # continuations first: each is one or a few tokens of a resident key
        cont, pool = self.cont, self.pool
        max_seqs = self.max_seqs if self.max_seqs is not None else 1 << 30
        cap = min(max_seqs, self.cont_cap)
        while cont and room > 0 and len(specs) < cap:
            task = cont[0]
            n = len(task.tokens)
            total = task.own_prefix + n
            if n > room:
                break
            if pool.tokens[task.key] < total and pool.grow(task.key, total) is None:
                self._evict(pool.pages_needed(total))
                if pool.grow(task.key, total) is None:
                    break
            cont.popleft()
            rows = tuple(task.readout_rows) if task.readout and task.readout_rows is not None else None
            specs.append(SeqSpec(task.reads, task.key, task.own_prefix, task.tokens, task.pos_start, task.readout,
                                 task, rows, task.full_readout, task.topk))
            task.done = n
            room -= n
        scanned = 0
        no_new = False
        stop = False
        # follow-ups (questions about resident documents) before new documents: they free
        # their documents' pages when answered, so under memory pressure the rows in flight
        # finish first instead of new documents taking the pages they need
        for dq in (self.follow, self.queue):
          deferred: list[Task] = []
          while dq and room > 0 and scanned < 4096 and not stop:
            if self.max_seqs is not None and len(specs) >= self.max_seqs:
                break
            task = dq.popleft()
            scanned += 1
            if not self._readable(task):
                deferred.append(task)
                continue
            total = task.own_prefix + len(task.tokens)
            if not self.pool.resident(task.key):
                if no_new:
                    deferred.append(task)
                    continue
                cap = total + (task.reserve_tokens if self.answer_headroom else 0)
                pages = self.pool.alloc(task.key, total, cap)
                if pages is None:
                    self._evict(self.pool.pages_needed(cap))
                    pages = self.pool.alloc(task.key, total, cap)
                if pages is None:
                    # keep new work in FIFO order under memory pressure, but
                    # still admit pieces of keys that are already resident
                    deferred.append(task)
                    no_new = True
                    continue
                for rk, _ in task.reads:
                    self.pool.borrow(task.key, rk)
            elif self.pool.tokens[task.key] < total:
                # a continuation (decode step, prefill piece) of a resident key
                if self.pool.grow(task.key, total) is None:
                    self._evict(self.pool.pages_needed(total))
                    if self.pool.grow(task.key, total) is None:
                        deferred.append(task)
                        stop = True
                        break
            piece = min(task.remaining, room)
            if task.bidirectional and piece < task.remaining:
                if task.remaining > self.chunk_tokens:
                    raise OversizedDocumentError(
                        f"a document-isolated block of {task.remaining} tokens does not fit one pass of "
                        f"{self.chunk_tokens} tokens")
                deferred.append(task)
                stop = True
                break
            if piece < task.remaining and piece < self.min_piece and specs:
                deferred.append(task)
                stop = True
                break
            if task.done == 0:
                self.stats.cached += sum(n for _, n in task.reads)
            last = piece == task.remaining
            rows = None
            readout = task.readout and last
            if task.readout and task.readout_rows is not None:
                # a task read at several rows reads, in each piece, the rows that fall in it
                rows = tuple(r - task.done for r in task.readout_rows if task.done <= r < task.done + piece)
                readout = bool(rows)
            specs.append(SeqSpec(reads=list(task.reads), own_key=task.key, own_start=task.own_prefix + task.done,
                                 tokens=task.tokens[task.done:task.done + piece],
                                 pos_start=task.pos_start + task.done, readout=readout, tag=task,
                                 readout_rows=rows if readout else None, full=task.full_readout, topk=task.topk,
                                 bidirectional=task.bidirectional))
            task.done += piece
            room -= piece
            if not last:
                deferred.append(task)  # the rest goes in a later chunk
                stop = True
                break
          # deferred tasks go back to the head of their queue in their original order
          for t in reversed(deferred):
              dq.appendleft(t)
        return specs

    # ------------------------------------------------------------ run
    def enable_graphs(self) -> None:
        """Run decode passes (one token per sequence) as CUDA graph replays (engine/graphs.py)."""
        if self.device.type == "cuda" and self.graphs is None:
            from quail_b200.engine.graphs import DecodeGraphs
            self.graphs = DecodeGraphs(self.model, self.arena, self.device)

    def _launch(self, specs: list[SeqSpec]):
        if self.nvtx:
            torch.cuda.nvtx.range_push(f"pass {self.stats.passes}: {len(specs)} seqs")
        try:
            self._launch_inner(specs)
        finally:
            if self.nvtx:
                torch.cuda.nvtx.range_pop()

    def _launch_inner(self, specs: list[SeqSpec]):
        ev0 = ev1 = None
        if self.gpu_timing:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        res = None
        if self.graphs is not None and self.graphs.eligible(specs):
            host, _ = self.packer.host_parts(specs)
            res = self.graphs.run(host, any(s.full and s.readout for s in specs),
                                  any(s.topk and s.readout for s in specs))
        if res is not None:
            logits, nbytes = res
            chunk = _Replayed(num_tokens=len(specs), upload_bytes=nbytes)
        else:
            chunk = self.packer.pack(specs)
            if getattr(chunk, "tree", None) is not None:
                self.stats.tree_passes += 1
            logits = self.model.forward_chunk(chunk, self.arena)
        if self.gpu_timing:
            ev1.record()
        for s in specs:
            self.written[s.own_key] = s.own_start + len(s.tokens)
        if self.device.type == "cuda" and logits is not None:
            host = torch.empty(logits.shape, dtype=logits.dtype, pin_memory=True)
            host.copy_(logits, non_blocking=True)
            done = torch.cuda.Event()
            done.record()
        else:
            host, done = logits, None
        self.stats.passes += 1
        self.stats.tokens += chunk.num_tokens
        self.stats.pass_tokens.append(chunk.num_tokens)
        self.stats.pass_rows.append(sum(1 for s in specs if s.readout and s.readout_rows is None))
        self.stats.h2d_bytes += chunk.upload_bytes
        if logits is not None:
            self.stats.d2h_bytes += logits.numel() * logits.element_size()
        if self.trace_dir is not None:
            pool = self.pool
            mem = torch.cuda.memory_allocated(self.device) if self.device.type == "cuda" else 0
            self.trace.append([round(time.perf_counter() - self._t_run, 6), self.stats.passes, chunk.num_tokens,
                               pool.free_pages, pool.num_pages - pool.free_pages, len(pool.owned),
                               len(getattr(pool, "retained", ()) or ()), int(mem)])
        self._inflight.append((specs, chunk, host, done, ev0, ev1))

    def _collect_one(self):
        specs, chunk, host, done, ev0, ev1 = self._inflight.popleft()
        if done is not None:
            done.synchronize()
        if ev0 is not None:
            self.stats.gpu_ms += ev0.elapsed_time(ev1)
        r = 0
        hnp = host.numpy() if hasattr(host, "numpy") else host   # one view for the whole pass
        for s in specs:
            task: Task = s.tag
            last = s.own_start + len(s.tokens) == task.own_prefix + len(task.tokens)
            row = None
            if s.readout:
                k = len(s.readout_rows) if s.readout_rows is not None else 1
                src = hnp if task.np_rows else host
                row = src[r] if s.readout_rows is None else src[r:r + k]
                r += k
                self.stats.readouts += 1
            if task.readout_rows is not None and task.readout:
                if row is not None:
                    task.got_rows.append(row.numpy().copy() if hasattr(row, "numpy") else np.array(row))
                if last:
                    row = np.concatenate(task.got_rows) if len(task.got_rows) != 1 else task.got_rows[0]
                    task.got_rows = []
            if last:
                if task.on_done:
                    task.on_done(task, row)
                if task.free_after:
                    self.free(task.key)

    def step(self) -> bool:
        """Launch one chunk if any task is admissible; collect finished chunks."""
        specs = self._admit()
        if specs:
            self._launch(specs)
            # keep one chunk queued behind the running one
            while len(self._inflight) > 1:
                self._collect_one()
            return True
        if self._inflight:
            self._collect_one()
            return True
        return False

    def run(self) -> ExecutorStats:
        t0 = time.perf_counter()
        self._t_run = t0
        self.trace = []
        try:
            return self._run(t0)
        finally:
            if self.trace_dir is not None and self.trace:
                self._write_trace()

    def _write_trace(self) -> None:
        import json
        os.makedirs(self.trace_dir, exist_ok=True)
        n = len([f for f in os.listdir(self.trace_dir) if f.startswith(f"headroom-{os.getpid()}-")])
        path = os.path.join(self.trace_dir, f"headroom-{os.getpid()}-{n}.json")
        with open(path, "w", encoding="utf-8") as f:
            json.dump({"columns": ["t_s", "pass", "tokens", "free_pages", "held_pages", "keys", "retained",
                                   "gpu_bytes"],
                       "num_pages": self.pool.num_pages, "page_tokens": self.pool.page_tokens,
                       "answer_admission": "headroom" if self.answer_headroom else "headroom=0",
                       "samples": self.trace}, f)

    def _run(self, t0: float) -> ExecutorStats:
        while self.pending() or self._inflight:
            if self.should_stop is not None and self.should_stop():
                self.abort()
                raise QueryCancelled("the query was stopped")
            if not self.step():
                if self.pending():
                    head = (self.follow or self.queue or self.cont)[0]
                    raise ArenaFullError(
                        f"{len(self.follow) + len(self.queue)} tasks cannot be admitted: {self.pool.free_pages} "
                        f"free pages; head {head.key!r} reads {head.reads}")
                break
        self.stats.wall_s += time.perf_counter() - t0
        return self.stats

    def pending(self) -> bool:
        """Tasks waiting for admission (new documents, follow-ups, continuations)."""
        return bool(self.queue or self.follow or self.cont)

    def abort(self) -> None:
        """Drop queued work, wait for in-flight passes, release every resident key."""
        self.queue.clear()
        self.follow.clear()
        self.cont.clear()
        while self._inflight:
            _, _, _, done, _, _ = self._inflight.popleft()
            if done is not None:
                done.synchronize()
        for key in list(self.pool.owned):
            self.pool.free_key(key)
        self.written.clear()
