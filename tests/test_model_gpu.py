"""Whole-model numerics: the kernel pipeline against the fp32 PyTorch model.

Both run the same packed chunks through the same executor; the fp32 model
uses the dequantized checkpoint weights, so the difference is activation
quantization (fp8 models) and bf16 rounding.
"""

import numpy as np
import pytest
import torch

from quail_b200 import ops
from quail_b200.engine.arena import KVArena
from quail_b200.engine.stage_executor import StageExecutor, Task
from quail_b200.models.config import QWEN3_GPU_TINY, QWEN3_GPU_TINY_GQA4
from quail_b200.models.qwen3 import Qwen3Pipeline, Qwen3Reference, Qwen3Weights
from quail_b200.models.weights import random_checkpoint

pytestmark = pytest.mark.gpu


def _run(model, cfg, prefix, docs, suffix, dtype):
    arena = KVArena(cfg.layers, 96, 128, cfg.num_kv_heads, cfg.head_dim, device="cuda", dtype=dtype)
    ex = StageExecutor(model, arena, 300, min_piece=16)
    got = {}
    ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
    for i, d in enumerate(docs):
        ex.submit(Task(key=i, tokens=np.concatenate([d, suffix]), pos_start=len(prefix), reads=[("p", len(prefix))],
                       readout=True, on_done=lambda t, row, i=i: got.__setitem__(i, row.float().cpu())))
    ex.run()
    return torch.stack([got[i] for i in range(len(docs))])


def _dist(a, b):
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("base,weight_dtype,layers", [(QWEN3_GPU_TINY, "fp8", 1), (QWEN3_GPU_TINY, "fp8", 2),
                                                      (QWEN3_GPU_TINY, "bf16", 2), (QWEN3_GPU_TINY_GQA4, "fp8", 2),
                                                      (QWEN3_GPU_TINY_GQA4, "bf16", 2)])
def test_pipeline_matches_fp32_model(base, weight_dtype, layers):
    # QWEN3_GPU_TINY_GQA4 runs the flagship layer sequence: MX fp8 GEMMs, the QKV epilogue with
    # norm + RoPE + KV write, and the persistent tcgen05 attention (4 q heads per KV head)
    cfg = base.with_(weight_dtype=weight_dtype, vocab=4096, max_position=8192, layers=layers)
    ckpt = random_checkpoint(cfg, seed=7, device="cuda")
    # non-trivial RMSNorm weights (random init leaves them at one): the fp8 pipeline folds
    # them into the projections it feeds, which this makes visible
    g = torch.Generator(device="cuda").manual_seed(3)
    for k in list(ckpt):
        if k.endswith("layernorm.weight") or k == "model.norm.weight":
            ckpt[k] = (ckpt[k].float() * (1 + 0.3 * torch.randn(ckpt[k].shape, generator=g, device="cuda"))).to(
                ckpt[k].dtype)
    ids = list(range(16))
    pipe = Qwen3Pipeline(cfg, Qwen3Weights(cfg, ckpt, "cuda", head_rows=ids))
    exact = Qwen3Reference(cfg, ckpt, device="cuda", head_rows=ids)
    emul = Qwen3Reference(cfg, ckpt, device="cuda", head_rows=ids, emulate_kernels=True)
    rng = np.random.default_rng(0)
    prefix = rng.integers(0, 4096, 48).astype(np.int32)
    docs = [rng.integers(0, 4096, n).astype(np.int32) for n in (10, 200, 64, 450, 129)]
    suffix = rng.integers(0, 4096, 24).astype(np.int32)
    got = _run(pipe, cfg, prefix, docs, suffix, torch.bfloat16)
    want = _run(exact, cfg, prefix, docs, suffix, torch.float32)
    close = _run(emul, cfg, prefix, docs, suffix, torch.float32)
    assert ops.read_and_clear_error(0) == 0
    d_kernel = _dist(got, want)
    d_emul = _dist(close, want)
    print(f"{cfg.name} {weight_dtype} L={layers}: kernel-vs-exact {d_kernel:.4f} emulated-vs-exact {d_emul:.4f} "
          f"kernel-vs-emulated {_dist(got, close):.4f}")
    # the kernels are as close to the exact fp32 model as an fp32 model that
    # rounds and quantizes at the same points
    assert d_kernel < 1.5 * d_emul + 0.02, (d_kernel, d_emul)
    agree = (got.argmax(1) == want.argmax(1)).float().mean().item()
    assert agree >= 0.6


def test_smoke_entry():
    from quail_b200.models.smoke import run_smoke
    run_smoke()


def test_sae_pipeline_matches_fp32_model():
    """SAE readout of the kernel pipeline vs the fp32 model rounding where the kernels round."""
    from quail_b200.models.config import QWEN3_GPU_SAE_TINY
    cfg = QWEN3_GPU_SAE_TINY.with_(vocab=4096, max_position=8192)
    ckpt = random_checkpoint(cfg, seed=5, device="cuda")
    pipe = Qwen3Pipeline(cfg, Qwen3Weights(cfg, ckpt, "cuda", head_rows=[0]))
    emul = Qwen3Reference(cfg, ckpt, device="cuda", head_rows=[0], emulate_kernels=True)
    rng = np.random.default_rng(2)
    prefix = rng.integers(0, 4096, 48).astype(np.int32)
    docs = [rng.integers(0, 4096, n).astype(np.int32) for n in (10, 200, 64, 129)]
    suffix = rng.integers(0, 4096, 12).astype(np.int32)
    got = _run(pipe, cfg, prefix, docs, suffix, torch.bfloat16)
    want = _run(emul, cfg, prefix, docs, suffix, torch.float32)
    assert ops.read_and_clear_error(0) == 0
    k = cfg.sae_keep
    for g, w in zip(got, want):
        gs = {int(i) for i, s in zip(g[:k], g[k:]) if s > 0}
        ws = {int(i) for i, s in zip(w[:k], w[k:]) if s > 0}
        assert len(gs & ws) >= 0.8 * max(len(ws), 1), (len(gs & ws), len(ws))
        top = min(len(ws), 8)
        assert torch.allclose(g[k:k + top], w[k:k + top], rtol=0.05, atol=0.05)
