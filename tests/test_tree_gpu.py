"""The tree attention path on the kernels: log-sum-exp output, the K7 merge, whole passes."""

import numpy as np
import pytest
import torch

from quail_b200 import ops
from quail_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp(min=1e-12)).item()


@pytest.fixture(autouse=True)
def _no_kernel_errors():
    torch.manual_seed(0)
    yield
    assert ops.read_and_clear_error(0) == 0


def test_persistent_attention_log_sum_exp():
    from test_kernels_gpu import _segmented_case
    specs = [(100, [48, 100]), (7, [48, 7]), (64, [48, 300, 64]), (130, [130]), (33, [200, 33])]
    q, kc, vc, seqs, pl = _segmented_case(64, specs, QH=8, KH=2, pages=1024)
    scale = ref.softmax_scale(128)
    want, want_lse = ref.segmented_attention_lse(q, kc, vc, seqs, pl, scale)
    lse = torch.empty(q.shape[0], 8, dtype=torch.float32, device=DEV)
    out = ops.prefill_attention_tc2(q, kc, vc, seqs.to(DEV), ref.attention_tiles(seqs, 64).to(DEV), pl.to(DEV),
                                    scale, fp8_out=False, lse=lse)
    assert rel_err(out, want) < 1e-2
    assert torch.allclose(lse, want_lse, atol=2e-2)


@pytest.mark.parametrize("fp8", [False, True])
def test_merge_kernel_against_fp32(fp8):
    T, R, QH = 300, 120, 8
    o_a = torch.randn(T, QH * 128, device=DEV).bfloat16()
    o_b = torch.randn(R, QH * 128, device=DEV).bfloat16()
    lse_a = torch.randn(T, QH, device=DEV) * 3
    lse_b = torch.randn(R, QH, device=DEV) * 3
    lse_b[5, 2] = float("-inf")
    source = torch.full((T,), -1, dtype=torch.int32, device=DEV)
    source[torch.randperm(T, device=DEV)[:R]] = torch.arange(R, dtype=torch.int32, device=DEV)
    want = ref.merge_lse(o_a, lse_a, o_b, lse_b, source)
    if fp8:
        o8, sf = ops.attention_merge(o_a, lse_a, o_b, lse_b, source, fp8_out=True)
        assert rel_err(ops.dequantize_mx(o8, sf), want) < 4e-2
    else:
        out = ops.attention_merge(o_a, lse_a, o_b, lse_b, source, fp8_out=False)
        assert rel_err(out, want) < 1e-2


def test_tree_and_unified_passes_agree_on_the_flagship_layers():
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.stage_executor import StageExecutor, Task
    from quail_b200.models.config import QWEN3_GPU_TINY_GQA4
    from quail_b200.models.qwen3 import Qwen3Pipeline, Qwen3Reference, Qwen3Weights
    from quail_b200.models.weights import random_checkpoint
    cfg = QWEN3_GPU_TINY_GQA4.with_(vocab=4096, max_position=8192)
    ckpt = random_checkpoint(cfg, seed=5, device=DEV)
    pipe = Qwen3Pipeline(cfg, Qwen3Weights(cfg, ckpt, DEV, head_rows=list(range(16))))
    rng = np.random.default_rng(3)
    anchor = rng.integers(0, 4096, 700).astype(np.int32)
    others = [rng.integers(0, 4096, n).astype(np.int32) for n in (20, 35, 9, 60, 14, 41, 1)]

    exact = Qwen3Reference(cfg, ckpt, device=DEV, head_rows=list(range(16)))

    def run(mode, model=pipe, dtype=torch.bfloat16):
        arena = KVArena(cfg.layers, 128, 128, cfg.num_kv_heads, 128, device=DEV, dtype=dtype)
        ex = StageExecutor(model, arena, 4096, min_piece=16, attention=mode)
        got = {}
        ex.submit(Task(key="a", tokens=anchor, pos_start=0, free_after=False))
        ex.run()
        for i, d in enumerate(others):
            ex.submit(Task(key=i, tokens=d, pos_start=700, reads=[("a", 700)], readout=True,
                           on_done=lambda t, row, i=i: got.__setitem__(i, row.float().cpu())))
        ex.run()
        return torch.stack([got[i] for i in range(len(others))]), ex.stats.tree_passes

    tree, n_tree = run("tree")
    unified, n_uni = run("unified")
    want, _ = run("unified", exact, torch.float32)
    assert n_tree == 1 and n_uni == 0
    # both paths round to fp8 at o_proj's input; the tree path also rounds each read to bf16
    # before the merge: it must be as close to the fp32 model as the unified path
    d_tree, d_uni = rel_err(tree, want), rel_err(unified, want)
    print(f"tree-vs-fp32 {d_tree:.4f} unified-vs-fp32 {d_uni:.4f} tree-vs-unified {rel_err(tree, unified):.4f}")
    assert d_tree < 1.3 * d_uni + 0.01, (d_tree, d_uni)
