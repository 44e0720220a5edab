"""Progress messages of a query's long steps, on the "quail" logger.

On a terminal each step is one line, and a running count (documents
answered in a region) is one bar updated in place with its rate and the
time left; detail messages (passes, tokens) are left out there. Anywhere
else (a log file, a worker's captured output) every message is one plain
line on stderr with a timestamp, details included, and a count logs a
line at each tenth of its total. Every line carries the run's tag (QUAIL_LOG_TAG, read
from the environment so worker processes inherit it) and this process's
GPU index when it has one.

Reference: quail/progress.py (the same two renderings, the GPU prefix and
the tag variable).
"""

from __future__ import annotations

import contextlib
import logging
import os
import sys
import time

LOG_TAG_ENV = "QUAIL_LOG_TAG"
LOGGER = "quail"

_gpu_index: int | None = None


def set_gpu_index(index: int | None) -> None:
    """Label this process's messages with its GPU index (worker processes)."""
    global _gpu_index
    _gpu_index = index


def _prefix() -> str:
    tag = os.environ.get(LOG_TAG_ENV)
    return ("" if not tag else f"[{tag}]") + ("" if _gpu_index is None else f"[GPU {_gpu_index}]")


def _terminal() -> bool:
    return bool(getattr(sys.stdout, "isatty", lambda: False)())


class _Handler(logging.Handler):
    def emit(self, record):
        text = self.format(record)
        if not _terminal():
            stamp = time.strftime("%m-%d %H:%M:%S", time.localtime(record.created))
            # plain lines go to stderr: stdout stays the caller's (a bench's JSON line, query output)
            print(f"{record.levelname} {stamp} [quail]{_prefix()} {text}", file=sys.stderr, flush=True)
            return
        if getattr(record, "detail", False):
            return
        mark = "✓" if getattr(record, "done", False) else "·"
        try:
            from rich.console import Console
            from rich.markup import escape
            Console(file=sys.stdout, highlight=False).print(f"  {mark} [dim]{escape(_prefix())}[/dim]{escape(text)}",
                                                           soft_wrap=True)
        except ImportError:
            print(f"  {mark} {_prefix()}{text}", file=sys.stdout, flush=True)


def logger() -> logging.Logger:
    log = logging.getLogger(LOGGER)
    if not any(isinstance(h, _Handler) for h in log.handlers):
        log.addHandler(_Handler())
        log.setLevel(logging.INFO)
        log.propagate = False
    return log


def say(message: str, *, detail: bool = False, done: bool = False) -> None:
    """One progress message: a step (shown everywhere) or a detail (log lines only)."""
    if os.environ.get("QUAIL_QUIET") == "1":
        return
    logger().info(message, extra={"detail": detail, "done": done})


class Count:
    """A running count toward a known total: a bar on a terminal, a line per tenth elsewhere."""

    def __init__(self, label: str, total: int, unit: str = ""):
        self.label, self.total, self.unit = label, max(int(total), 0), unit
        self.done = 0
        self.t0 = time.perf_counter()
        self._next_tenth = 1
        self._bar = None
        self._task = None
        if _terminal() and os.environ.get("QUAIL_QUIET") != "1":
            try:
                from rich.progress import BarColumn, Progress, TaskProgressColumn, TextColumn, TimeRemainingColumn
                self._bar = Progress(TextColumn(f"  {_prefix()}{label}"), BarColumn(), TaskProgressColumn(),
                                     TimeRemainingColumn(), transient=True)
                self._bar.start()
                self._task = self._bar.add_task(label, total=self.total)
            except ImportError:
                self._bar = None

    def advance(self, n: int = 1) -> None:
        self.done += n
        if self._bar is not None:
            self._bar.update(self._task, completed=self.done)
            return
        while self.total and self._next_tenth <= 10 and self.done * 10 >= self._next_tenth * self.total:
            rate = self.done / max(time.perf_counter() - self.t0, 1e-9)
            say(f"{self.label}: {self.done}/{self.total}{self.unit} ({rate:.1f}/s)", detail=True)
            self._next_tenth += 1

    def close(self) -> None:
        if self._bar is not None:
            self._bar.stop()
            self._bar = None
        dt = time.perf_counter() - self.t0
        say(f"{self.label}: {self.done}{self.unit} in {dt:.2f}s", done=True)


@contextlib.contextmanager
def count(label: str, total: int, unit: str = ""):
    c = Count(label, total, unit)
    try:
        yield c
    finally:
        c.close()
