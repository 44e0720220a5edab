"""Device spec lines from validated GEMM calibration summaries.

    python -m quail_b200.calibrate.to_spec calibration/b200 [more summaries or directories]

Prints `mamf_fp8_flops = ...` and `mamf_bf16_flops = ...` (FLOP/s, the highest
validated MAMF of each precision over the summaries) for the device's TOML file;
the cost model prices GEMM work at them where present (the reference's
calibrate/to_spec.py).
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

from quail_b200.calibrate.gemm import PRECISIONS, validate_clocks


def load(paths) -> list[dict]:
    out = []
    for p in map(Path, paths):
        files = sorted(p.rglob("summary.json")) if p.is_dir() else [p]
        out.extend(json.loads(f.read_text()) for f in files)
    if not out:
        raise ValueError("no calibration summaries found")
    return out


def spec_lines(summaries: list[dict]) -> str:
    """The best MAMF of each precision, as spec lines.

    Raises:
        ValueError: summaries of several devices, an unvalidated run, or a bad rate.
    """
    devices = {s.get("device") for s in summaries}
    if len(devices) != 1:
        raise ValueError(f"summaries of one device only, not {sorted(map(str, devices))}")
    best: dict = {}
    for s in summaries:
        validate_clocks(s.get("clocks") or {})
        for p, r in (s.get("runs") or {}).items():
            if p not in PRECISIONS:
                raise ValueError(f"unknown precision {p!r}")
            t = float((r.get("mamf") or {}).get("tflops", 0))
            if not math.isfinite(t) or t <= 0:
                raise ValueError(f"invalid {p} MAMF {t}")
            best[p] = max(best.get(p, 0.0), t * 1e12)
    return "\n".join(f"mamf_{p}_flops = {best[p]:.6g}" for p in PRECISIONS if p in best)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("paths", nargs="+")
    print(spec_lines(load(ap.parse_args(argv).paths)))


if __name__ == "__main__":
    main()
