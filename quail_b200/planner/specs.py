"""Device specs: the peaks the cost model prices work against.

B200 numbers: nominal dense peaks (bf16 2.25, fp8 4.5, fp4 9 PFLOP/s),
8 TB/s HBM3e, 180 GB; the reference's spec has the same
(quail/specs/data/devices/b200.toml:2-8). `measured_b200()` swaps in the
pool's measured copy bandwidth and cuBLAS bf16 throughput when the
driver-written MEASURED_PEAKS.json sits at the repository root.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, replace


@dataclass(frozen=True)
class DeviceSpec:
    name: str
    mem_bytes: float
    hbm_bw: float
    fp8_flops: float
    bf16_flops: float
    fp4_flops: float = 0.0
    page_tokens: int = 128
    usd_per_hour: float = 0.0
    sms: int = 0


DEVICES = {
    "b200": DeviceSpec("b200", mem_bytes=183_359 * 2**20, hbm_bw=8e12, fp8_flops=4.5e15, bf16_flops=2.25e15,
                       fp4_flops=9e15, page_tokens=128, usd_per_hour=6.2496, sms=148),
    "h100-sxm": DeviceSpec("h100-sxm", mem_bytes=85_520_809_984, hbm_bw=3.35e12, fp8_flops=1.629e15,
                           bf16_flops=0.857e15, page_tokens=16),
    "cpu": DeviceSpec("cpu", mem_bytes=8 << 30, hbm_bw=50e9, fp8_flops=1e12, bf16_flops=1e12, page_tokens=16),
}


def measured_b200(path: str | None = None) -> DeviceSpec:
    path = path or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                "MEASURED_PEAKS.json")
    spec = DEVICES["b200"]
    try:
        with open(path) as f:
            m = json.load(f)
    except (OSError, ValueError):
        return spec
    return replace(spec, hbm_bw=float(m.get("hbm_gbs", spec.hbm_bw / 1e9)) * 1e9,
                   bf16_flops=float(m.get("bf16_tflops", spec.bf16_flops / 1e12)) * 1e12)
