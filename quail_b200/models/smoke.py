"""One tiny packed-prefill forward + yes/no readout of the flagship pipeline on cuda:0.

The model is the flagship's layer sequence at the smallest size (fp8 MX GEMMs,
the QKV epilogue with q/k norm + RoPE + KV write, the persistent tcgen05
attention with 4 q heads per KV head).
"""

from __future__ import annotations

import numpy as np
import torch


def run_smoke() -> None:
    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor
    from quail_b200.models.build import build_pipeline
    from quail_b200.models.config import QWEN3_GPU_TINY_GQA4

    assert torch.cuda.is_available(), "smoke needs a GPU"
    ops.native()
    cfg = QWEN3_GPU_TINY_GQA4
    dev = torch.device("cuda", 0)
    pipe = build_pipeline(cfg, device=dev, seed=0, answer_ids=(1, 2, 3, 4))
    arena = KVArena(cfg.layers, 64, 128, cfg.num_kv_heads, cfg.head_dim, device=dev)
    rng = np.random.default_rng(0)
    prefix = rng.integers(0, 1000, 48).astype(np.int32)
    docs = [rng.integers(0, 1000, n).astype(np.int32) for n in (100, 37, 250)]
    call = Call(kind="score", suffix=rng.integers(0, 1000, 20).astype(np.int32), true_cols=[0, 1],
                false_cols=[2, 3], name="s")
    ex = StageExecutor(pipe, arena, 512)
    res = RegionRun(ex, prefix, docs, [call]).run()
    torch.cuda.synchronize()
    assert ops.read_and_clear_error(0) == 0
    vals = [r.values["s"] for r in res]
    assert all(np.isfinite(v) and 0.0 <= v <= 1.0 for v in vals), vals
    print("smoke ok", vals, "passes", ex.stats.passes)


if __name__ == "__main__":
    run_smoke()
