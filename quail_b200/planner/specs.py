"""Device specs: the peaks the cost model prices work against.

Read from the TOML device specs (quail_b200/specs/data/devices: b200,
h100-sxm, l40s, rtx-pro-6000-blackwell-server; the reference's spec format).
B200: nominal dense peaks (bf16 2.25, fp8 4.5, fp4 9 PFLOP/s), 8 TB/s HBM3e. `measured_b200()` swaps in the
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
    fp32_flops: float = 0.0
    cuda_name: str = ""
    # measured burst matmul rates (quail_b200.calibrate), 0 = use the nominal peaks
    mamf_fp8_flops: float = 0.0
    mamf_bf16_flops: float = 0.0

    def gemm_flops(self, fp8: bool) -> float:
        """The rate GEMM work is priced at: the calibrated MAMF where measured, else the peak."""
        if fp8:
            return self.mamf_fp8_flops or self.fp8_flops
        return self.mamf_bf16_flops or self.bf16_flops


def _devices() -> dict:
    """The TOML device specs (quail_b200/specs/data/devices) plus the host CPU."""
    from quail_b200.specs.loading import builtin_devices
    out = builtin_devices()
    out["cpu"] = DeviceSpec("cpu", mem_bytes=8 << 30, hbm_bw=50e9, fp8_flops=1e12, bf16_flops=1e12, page_tokens=16)
    return out


DEVICES = _devices()


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
