"""Decode passes as CUDA graph replays: same tokens as the eager passes."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(pipe, arena, graphs, rows=40, max_new=12):
    from quail_b200.engine.region import Call, RegionRun
    from quail_b200.engine.stage_executor import StageExecutor
    from quail_b200.utils.synthetic import make_workload
    wl = make_workload(rows, median=60, sigma=0.6, hi=300, suffix_tokens=12, seed=7)
    wl.bodies = [b % 4000 for b in wl.bodies]
    ex = StageExecutor(pipe, arena, 2048)
    if graphs:
        ex.enable_graphs()
    call = Call(kind="map", suffix=wl.suffix % 4000, max_tokens=max_new, stop_ids=(), name="map")
    run = RegionRun(ex, wl.prefix % 4000, wl.bodies, [call], answer_width=8)
    res = run.run()
    return [r.values["map"] for r in res], ex


@pytest.mark.parametrize("model", ["qwen3-gpu-tiny"])
def test_graph_replays_match_eager(model):
    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.build import build_pipeline
    from quail_b200.models.config import MODEL_CONFIGS
    cfg = MODEL_CONFIGS[model]
    dev = torch.device("cuda", 0)
    pipe = build_pipeline(cfg, dev, answer_ids=list(range(8)))
    arena = KVArena(cfg.layers, 512, 128, cfg.num_kv_heads, cfg.head_dim, device=dev)
    eager, _ = _run(pipe, arena, False)
    n0 = ops.launch_count()
    graphed, ex = _run(pipe, arena, True)
    assert ex.graphs.captures >= 1 and ex.graphs.replays >= 1
    assert ops.launch_count() > n0
    assert ops.read_and_clear_error(0) == 0
    assert all(len(g) == 12 for g in graphed)
    assert graphed == eager


@pytest.mark.parametrize("model", ["qwen3.5-gpu-tiny", "lfm2-gpu-tiny"])
def test_hybrid_graph_replays_match_eager(model):
    """Hybrids: the token mixers' decode step reads and writes its state slots through the
    graph's state_io rows; padding rows start from zeros and write no state."""
    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.build import build_pipeline
    from quail_b200.models.config import MODEL_CONFIGS
    cfg = MODEL_CONFIGS[model]
    dev = torch.device("cuda", 0)
    pipe = build_pipeline(cfg, dev, answer_ids=list(range(8)))

    def arena():
        return KVArena.for_model(cfg, 512, 128, device=dev, dtype=torch.bfloat16, state_slots=96)
    eager, _ = _run(pipe, arena(), False, rows=37)
    graphed, ex = _run(pipe, arena(), True, rows=37)
    assert ex.graphs.captures >= 1 and ex.graphs.replays >= 1
    assert ops.read_and_clear_error(0) == 0
    assert all(len(g) == 12 for g in graphed)
    assert graphed == eager
