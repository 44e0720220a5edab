"""GEMM calibration: validation of measured rates and the spec lines they become."""

import json

import pytest

from quail_b200.calibrate.gemm import best_of, rate_tflops, summarize, validate_clocks
from quail_b200.calibrate.to_spec import load, spec_lines
from quail_b200.planner.budgets import Budgets
from quail_b200.planner.specs import DeviceSpec

GOOD = {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 40}


def test_rates_and_the_best_shape():
    assert rate_tflops(8192, 8192, 8192, 1.0) == pytest.approx(2 * 8192 ** 3 / 1e-3 / 1e12)
    best = best_of({"cublas": {"a": 1500.0, "b": 1580.5}, "qb_tcgen05": {"a": 1602.0}})
    assert best == {"tflops": 1602.0, "shape": "a", "impl": "qb_tcgen05"}


def test_clock_validation_refuses_slow_or_throttled_runs():
    validate_clocks(GOOD)
    with pytest.raises(ValueError, match="samples"):
        validate_clocks({"samples": 0})
    with pytest.raises(ValueError, match="thermal"):
        validate_clocks(dict(GOOD, reasons=["hw_thermal_slowdown"]))
    with pytest.raises(ValueError, match="0.97"):
        validate_clocks(dict(GOOD, sm_mhz=1500.0))


def test_summaries_become_spec_lines_and_price_the_gemms(tmp_path):
    m1 = summarize("b200", {"rates": {"fp8": {"qb_mx": {"s": 2900.0}}, "bf16": {"cublas": {"s": 1590.0}}},
                            "clocks": GOOD})
    m2 = summarize("b200", {"rates": {"fp8": {"cublaslt": {"s": 2950.0}}}, "clocks": GOOD})
    for i, m in enumerate((m1, m2)):
        d = tmp_path / f"run{i}"
        d.mkdir()
        (d / "summary.json").write_text(json.dumps(m))
    text = spec_lines(load([tmp_path]))
    assert text.splitlines() == ["mamf_fp8_flops = 2.95e+15", "mamf_bf16_flops = 1.59e+15"]
    with pytest.raises(ValueError, match="one device"):
        spec_lines([m1, dict(m2, device="h100-sxm")])
    # the cost model prices GEMM work at the calibrated rate where a device has one
    from quail_b200.models.config import QWEN3_4B
    nominal = DeviceSpec("x", mem_bytes=180e9, hbm_bw=7.7e12, fp8_flops=4.5e15, bf16_flops=2.25e15)
    measured = DeviceSpec("x", mem_bytes=180e9, hbm_bw=7.7e12, fp8_flops=4.5e15, bf16_flops=2.25e15,
                          mamf_fp8_flops=2.95e15)
    a = Budgets(QWEN3_4B, nominal, 16384).pass_seconds(16384, 200)
    b = Budgets(QWEN3_4B, measured, 16384).pass_seconds(16384, 200)
    assert b == pytest.approx(a * 4.5 / 2.95, rel=1e-6)
