"""Run-twice determinism: a kernel without atomics in its sums gives bitwise-equal outputs on
the same inputs, and a whole pass through a model gives bitwise-equal readouts.

The reference's race checks are bitwise-equality tests of launch variants
(tests/gpu/test_decode_evaluator.py:36,116); here the same discipline covers
the kernels whose reductions run in a fixed order (the GEMMs accumulate in TMEM
in K order; the attention kernels' softmax order is fixed per tile; the
residual norm's partial sums are per column block, with no atomics).
"""

import numpy as np
import pytest
import torch

from quail_b200 import ops
from quail_b200.engine.arena import KVArena
from quail_b200.engine.stage_executor import StageExecutor, Task
from quail_b200.models.weights import random_checkpoint
from quail_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_kernel_errors():
    torch.manual_seed(0)
    yield
    assert ops.read_and_clear_error(0) == 0


def test_gemms_are_bitwise_repeatable():
    M, N, K = 1000, 2560, 4096
    a = torch.randn(M, K, device=DEV).bfloat16()
    w = torch.randn(N, K, device=DEV) * 0.02
    a8, asf = ops.quantize_act_mx(a.float())
    w8, wsf = ops.quantize_weight_mx(w)
    outs = [ops.gemm_mx(a8, asf, w8, wsf) for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    wb = w.bfloat16()
    bf = [ops.gemm(a, wb) for _ in range(2)]
    assert torch.equal(bf[0], bf[1])


def test_attention_kernels_are_bitwise_repeatable():
    from test_kernels_gpu import _segmented_case
    specs = [(100, [48, 100]), (7, [48, 7]), (64, [48, 300, 64]), (300, [48, 300]), (1, [48, 1])]
    q, kc, vc, seqs, pl = _segmented_case(128, specs, QH=8, KH=2, pages=1024)
    scale = ref.softmax_scale(128)
    sd, pld = seqs.to(DEV), pl.to(DEV)
    blocks = ref.attention_tiles(seqs, 64).to(DEV)
    a = [ops.prefill_attention_tc2(q, kc, vc, sd, blocks, pld, scale, fp8_out=False) for _ in range(2)]
    assert torch.equal(a[0], a[1])
    tiles = ref.attention_tiles(seqs).to(DEV)
    b = [ops.prefill_attention_tc(q, kc, vc, sd, tiles, pld, scale, fp8_out=False) for _ in range(2)]
    assert torch.equal(b[0], b[1])


def _pass(model, cfg, arena_fn):
    arena = arena_fn()
    ex = StageExecutor(model, arena, 512, min_piece=16)
    got = {}
    rng = np.random.default_rng(5)
    prefix = rng.integers(0, 4096, 48).astype(np.int32)
    docs = [rng.integers(0, 4096, n).astype(np.int32) for n in (10, 300, 64, 129)]
    suffix = rng.integers(0, 4096, 16).astype(np.int32)
    ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
    for i, d in enumerate(docs):
        ex.submit(Task(key=i, tokens=np.concatenate([d, suffix]), pos_start=48, reads=[("p", 48)], readout=True,
                       on_done=lambda t, row, i=i: got.__setitem__(i, row.float().cpu())))
    ex.run()
    return torch.stack([got[i] for i in range(len(docs))])


@pytest.mark.parametrize("name", ["qwen3-gpu-tiny-gqa4", "qwen3.5-gpu-tiny", "qwen3.5-gpu-tiny-fp8"])
def test_a_model_pass_is_bitwise_repeatable(name):
    from quail_b200.models.config import MODEL_CONFIGS
    cfg = MODEL_CONFIGS[name].with_(vocab=4096, max_position=8192)
    ckpt = random_checkpoint(cfg, seed=2, device=DEV)
    ids = list(range(16))
    if cfg.is_hybrid:
        from quail_b200.models.qwen3_5_gpu import Qwen35Pipeline
        model = Qwen35Pipeline(cfg, ckpt, DEV, head_rows=ids)

        def arena_fn():
            return KVArena.for_model(cfg, 64, 16, device=DEV, dtype=torch.bfloat16, state_slots=16)
    else:
        from quail_b200.models.qwen3 import Qwen3Pipeline, Qwen3Weights
        model = Qwen3Pipeline(cfg, Qwen3Weights(cfg, ckpt, DEV, head_rows=ids))

        def arena_fn():
            return KVArena(cfg.layers, 64, 128, cfg.num_kv_heads, cfg.head_dim, device=DEV)
    first = _pass(model, cfg, arena_fn)
    again = _pass(model, cfg, arena_fn)
    assert torch.equal(first, again)
