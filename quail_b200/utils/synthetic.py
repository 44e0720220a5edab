"""Synthetic document tables of the benchmark configurations.

Bodies are random token ids uniform in [0, 151643) with lognormal lengths
(median m, sigma s) clipped to [lo, hi], seeded; the shared instruction
prefix and the question suffix are fixed seeded token runs of the stated
lengths. This is the shape of the AI.IF workloads in the benchmark configs:
a 48-token template prefix reused by every row, a ~16-token instruction.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

TOKEN_HIGH = 151_643


@dataclass
class Workload:
    prefix: np.ndarray
    suffix: np.ndarray
    bodies: list

    @property
    def rows(self) -> int:
        return len(self.bodies)

    def row_tokens(self, i: int) -> int:
        return len(self.prefix) + len(self.bodies[i]) + len(self.suffix)

    def fresh_tokens(self) -> int:
        return len(self.prefix) + sum(len(b) + len(self.suffix) for b in self.bodies)

    def prompt_tokens(self) -> int:
        """Every prompt's full length, the shared prefix counted each time."""
        return sum(self.row_tokens(i) for i in range(self.rows))


def lognormal_lengths(n: int, median: float, sigma: float, lo: int, hi: int, rng) -> np.ndarray:
    return np.clip(np.round(median * np.exp(sigma * rng.standard_normal(n))), lo, hi).astype(np.int64)


def make_workload(rows: int, *, median: float = 180, sigma: float = 0.6, lo: int = 16, hi: int = 2048,
                  prefix_tokens: int = 48, suffix_tokens: int = 40, seed: int = 0) -> Workload:
    rng = np.random.default_rng(seed)
    fixed = np.random.default_rng(12345)  # the template is the same on every rank
    prefix = fixed.integers(0, TOKEN_HIGH, prefix_tokens).astype(np.int32)
    suffix = fixed.integers(0, TOKEN_HIGH, suffix_tokens).astype(np.int32)
    lens = lognormal_lengths(rows, median, sigma, lo, hi, rng)
    bodies = [rng.integers(0, TOKEN_HIGH, int(n)).astype(np.int32) for n in lens]
    return Workload(prefix=prefix, suffix=suffix, bodies=bodies)


def rows_for_tokens(tokens: int, median: float = 180, sigma: float = 0.6, suffix_tokens: int = 40) -> int:
    mean = median * float(np.exp(sigma * sigma / 2)) + suffix_tokens
    return int(tokens / mean) + 1
