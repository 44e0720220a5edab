"""Measure MAMF, the maximum achievable matmul rate in short bursts, per precision.

    python -m quail_b200.calibrate.gemm --device b200 [--precision fp8,bf16] [--out calibration]

The reference runs an external finder script on cuBLAS (calibrate/gemm.py,
calibrate/README.md) and copies the best rate into its device specs. Here the
search runs in-process over a grid of GEMM shapes, on both the library GEMM
(cuBLAS `torch.mm` for bf16, cuBLASLt `torch._scaled_mm` for fp8) and this
engine's own tcgen05 kernels (the bf16 GEMM and the MX block-scaled fp8 GEMM),
and records the best rate of each:

  - every shape: a few warm-up launches, then bursts of launches timed with CUDA
    events on the launching stream; a shape's rate is its best burst;
  - the SM clock and throttle reasons are sampled (nvidia-smi) during the
    search; a run whose median loaded clock is under 0.97 x the GPU's maximum,
    or that saw a thermal or hardware slowdown, is not a MAMF and is refused;
  - the summary (`<out>/<device>/gemm/<stamp>/summary.json`) keeps every shape's
    rate per implementation, the best one, and the clocks.

quail_b200.calibrate.to_spec turns summaries into `mamf_fp8_flops` /
`mamf_bf16_flops` lines for a device spec file; the cost model prices GEMM
work at those rates where a device has them.
"""

from __future__ import annotations

import argparse
import json
import os
import time

PRECISIONS = ("fp8", "bf16")
# the search grid: M (tokens) x N x K; the model widths of the flagship family and
# square sizes around the library's sweet spot
SHAPES = tuple((m, n, k) for m in (4096, 8192, 16384) for n, k in
               ((6144, 2560), (2560, 4096), (19456, 2560), (2560, 9728), (8192, 8192), (16384, 16384)))
SLOWDOWNS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


def rate_tflops(m: int, n: int, k: int, ms: float) -> float:
    return 2.0 * m * n * k / (ms * 1e-3) / 1e12


def validate_clocks(clocks: dict) -> None:
    """Refuse a measurement that was not taken at the boost clock.

    Raises:
        ValueError: no clock samples, a slowdown reason, or a median SM clock under
            0.97 x the maximum.
    """
    if not clocks or not clocks.get("samples"):
        raise ValueError("no SM clock samples: a MAMF must be measured at a validated clock")
    bad = [r for r in clocks.get("reasons", []) if r in SLOWDOWNS]
    if bad:
        raise ValueError(f"the clock slowed down during the search ({', '.join(bad)})")
    mhz, top = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    if not mhz or not top or mhz < 0.97 * top:
        raise ValueError(f"median SM clock {mhz} MHz is under 0.97 x the maximum {top} MHz")


def best_of(rates: dict) -> dict:
    """The best shape and rate over every implementation of one precision."""
    best = {"tflops": 0.0}
    for impl, shapes in rates.items():
        for shape, tflops in shapes.items():
            if tflops > best["tflops"]:
                best = {"tflops": tflops, "shape": shape, "impl": impl}
    return best


def _time(fn, warmup: int, bursts: int, per_burst: int) -> float:
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(bursts):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(per_burst):
            fn()
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e) / per_burst)
    return best


def _cases(precision: str, m: int, n: int, k: int):
    """(implementation name, zero-argument GEMM) pairs for one shape."""
    import torch

    from quail_b200 import ops
    dev = "cuda"
    a = torch.randn(m, k, device=dev)
    b = torch.randn(n, k, device=dev) * 0.02
    if precision == "bf16":
        ab, bb = a.bfloat16(), b.bfloat16()
        bt = bb.t()
        return [("cublas", lambda: torch.mm(ab, bt)), ("qb_tcgen05", lambda: ops.gemm(ab, bb))]
    a8, sfa = ops.quantize_act_mx(a)
    b8, sfb = ops.quantize_weight_mx(b)
    one = torch.ones((), device=dev)
    at8 = a.to(torch.float8_e4m3fn)
    bt8 = b.to(torch.float8_e4m3fn).t()
    return [("cublaslt", lambda: torch._scaled_mm(at8, bt8, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)),
            ("qb_mx", lambda: ops.gemm_mx(a8, sfa, b8, sfb))]


def measure(precisions=PRECISIONS, shapes=SHAPES, warmup: int = 3, bursts: int = 5, per_burst: int = 10) -> dict:
    """Every shape's best burst rate per implementation, with the clocks seen."""
    import torch

    from quail_b200.utils.clocks import ClockSampler
    sampler = ClockSampler(torch.cuda.current_device()).start()
    rates: dict = {}
    try:
        for p in precisions:
            rates[p] = {}
            for m, n, k in shapes:
                for impl, fn in _cases(p, m, n, k):
                    ms = _time(fn, warmup, bursts, per_burst)
                    rates[p].setdefault(impl, {})[f"{m}x{n}x{k}"] = round(rate_tflops(m, n, k, ms), 1)
                torch.cuda.empty_cache()
    finally:
        clocks = sampler.stop()
    return {"rates": rates, "clocks": clocks}


def summarize(device: str, measured: dict, gpu_name: str = "") -> dict:
    """The summary a run writes: per precision its MAMF, with every rate kept.

    Raises:
        ValueError: the clocks do not validate the run (validate_clocks).
    """
    validate_clocks(measured["clocks"])
    runs = {}
    for p, impls in measured["rates"].items():
        runs[p] = {"rates": impls, "mamf": best_of(impls)}
    return {"device": device, "gpu": gpu_name, "clocks": measured["clocks"], "runs": runs}


def run(device: str, out: str, precisions=PRECISIONS, shapes=SHAPES) -> dict:
    import torch
    stamp = time.strftime("%Y%m%dT%H%M%SZ", time.gmtime())
    measured = measure(precisions, shapes)
    summary = summarize(device, measured, torch.cuda.get_device_name())
    path = os.path.join(out, device, "gemm", stamp)
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "summary.json"), "w") as f:
        json.dump(summary, f, indent=2)
    return summary


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="measure GEMM MAMF per precision")
    ap.add_argument("--device", default="b200")
    ap.add_argument("--precision", default="fp8,bf16")
    ap.add_argument("--out", default="calibration")
    ap.add_argument("--quick", action="store_true", help="three shapes only")
    args = ap.parse_args(argv)
    shapes = SHAPES[-3:] if args.quick else SHAPES
    summary = run(args.device, args.out, tuple(args.precision.split(",")), shapes)
    for p, r in summary["runs"].items():
        m = r["mamf"]
        print(f"{args.device} {p}: MAMF {m['tflops']} TFLOPS ({m.get('impl')}, {m.get('shape')})", flush=True)


if __name__ == "__main__":
    main()
