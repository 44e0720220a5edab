"""Speed-of-light estimate of a query's model work on the configured GPUs.

The reference reports the time the AI calls would take at the device's peak
(quail/api/sol.py:365): prompt tokens times two FLOPs per active parameter
over the tensor peak, or the weight and KV bytes over HBM bandwidth,
whichever is slower, divided over the model copies.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class SpeedOfLightEstimate:
    seconds: float
    compute_seconds: float
    memory_seconds: float
    tokens: int
    gpus: int


def speed_of_light_estimate(config, prompt_tokens: int, mean_context_tokens: float = 0.0) -> SpeedOfLightEstimate:
    from quail_b200.api.config import check_config
    from quail_b200.planner.budgets import Budgets, weight_bytes
    cfg = check_config(config)
    b = Budgets.for_model(cfg, config.device, gpus=config.gpus)
    peak = b.device.fp8_flops if cfg.fp8 else b.device.bf16_flops
    flops = 2.0 * cfg.dense_params_per_token() * prompt_tokens + 4.0 * cfg.layers * cfg.q_dim * mean_context_tokens \
        * prompt_tokens
    compute = flops / peak / config.gpus
    passes = max(1, -(-prompt_tokens // b.chunk_tokens))
    memory = (weight_bytes(cfg) * passes / config.gpus + prompt_tokens * cfg.kv_bytes_per_token()) / b.device.hbm_bw
    return SpeedOfLightEstimate(seconds=max(compute, memory), compute_seconds=compute, memory_seconds=memory,
                                tokens=prompt_tokens, gpus=config.gpus)
