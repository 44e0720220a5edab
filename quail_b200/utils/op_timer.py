"""Device time per named op, from CUDA event pairs on the current stream.

Enabled with QB_OP_TIMING=1 (off by default: recording events adds a little
host work). Events are read only in `summary()`, after a synchronize, so the
timed ops run as they would untimed. For multi-GPU runs each rank reports
its own sums; waits on peers appear inside the op that waits.
"""

from __future__ import annotations

import os
from collections import defaultdict
from contextlib import contextmanager

import torch


class OpTimer:
    def __init__(self, enabled: bool | None = None):
        self.enabled = os.environ.get("QB_OP_TIMING") == "1" if enabled is None else enabled
        self._events: list = []

    @contextmanager
    def __call__(self, name: str):
        if not self.enabled:
            yield
            return
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        yield
        b.record()
        self._events.append((name, a, b))

    def reset(self) -> None:
        self._events.clear()

    def summary(self) -> dict:
        """{op: [ms total, count]} since the last reset (synchronizes)."""
        if not self._events:
            return {}
        torch.cuda.synchronize()
        out: dict = defaultdict(lambda: [0.0, 0])
        for name, a, b in self._events:
            out[name][0] += a.elapsed_time(b)
            out[name][1] += 1
        self._events.clear()
        return {k: [round(v[0], 3), v[1]] for k, v in out.items()}
