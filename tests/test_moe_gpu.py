"""MoE kernels (route, plan, dispatch + grouped gate_up, down + combine push,
combine + norm) against the fp32 PyTorch statement, on one GPU (W = 1)."""

import numpy as np
import pytest
import torch

from quail_b200 import ops
from quail_b200.models.config import QWEN3_MOE_GPU_TINY
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


@pytest.mark.parametrize("M,E,K", [(1, 16, 4), (300, 16, 4), (1000, 128, 8), (77, 256, 8)])
def test_moe_route(M, E, K):
    C = ops.native()
    logits = torch.randn(M, E, device=DEV).bfloat16()
    ids = torch.zeros(M * K, dtype=torch.int32, device=DEV)
    wts = torch.zeros(M * K, dtype=torch.float32, device=DEV)
    pos = torch.zeros(M * K, dtype=torch.int32, device=DEV)
    counts = torch.zeros(E, dtype=torch.int32, device=DEV)
    C.moe_route(logits, E, K, ids, wts, pos, counts)
    rid, rw = ref.moe_route(logits.float(), K)
    got_ids = ids.view(M, K).long()
    # same weights in the same (descending) order; at exact ties (bf16 logits
    # tie often) any of the tied experts is a valid pick
    assert torch.allclose(wts.view(M, K), rw, atol=1e-5)
    probs = torch.softmax(logits.float(), dim=-1)
    top = probs.topk(K, dim=-1).values
    assert torch.allclose(probs.gather(1, got_ids), top, atol=1e-6)
    assert torch.equal(got_ids.sort(1).values.unique_consecutive(dim=1).shape[1] * torch.ones(1), K * torch.ones(1))
    # slots: for each expert, positions 0..count-1 each used once
    assert torch.equal(counts.cpu(), torch.bincount(got_ids.flatten().cpu(), minlength=E).int())
    for e in range(E):
        p = pos[ids == e].sort().values.cpu()
        assert torch.equal(p, torch.arange(p.numel(), dtype=torch.int32))


def _layer(cfg, seed=0):
    from quail_b200.ops.quant import interleave_gate_up_mx, quantize_weight_mx
    g = torch.Generator(device=DEV).manual_seed(seed)
    E, H, I = cfg.num_experts, cfg.hidden, cfg.moe_intermediate
    L = {"router": (torch.randn(E, H, generator=g, device=DEV) * H ** -0.5).bfloat16()}
    gu, gus, d, ds, ex = [], [], [], [], []
    for _ in range(E):
        wg = torch.randn(I, H, generator=g, device=DEV) * 0.02
        wu = torch.randn(I, H, generator=g, device=DEV) * 0.02
        wd = torch.randn(H, I, generator=g, device=DEV) * 0.02
        q, s = interleave_gate_up_mx(torch.cat([wg, wu]))
        gu.append(q)
        gus.append(s)
        q2, s2 = quantize_weight_mx(wd)
        d.append(q2)
        ds.append(s2)
        # the exact values the kernels multiply
        qg, sg = quantize_weight_mx(wg)
        qu, su = quantize_weight_mx(wu)
        ex.append((ops.dequantize_mx(qg, sg), ops.dequantize_mx(qu, su), ops.dequantize_mx(q2, s2)))
    L.update(wgu=torch.cat(gu), sgu=torch.cat(gus), wd=torch.cat(d), sd=torch.cat(ds))
    return L, ex


def _moe_ref(x, ids, wts, ex):
    out = torch.zeros_like(x)
    for e, (wg, wu, wd) in enumerate(ex):
        rows, ks = (ids == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        a = ref.silu_mul(x[rows] @ wg.t(), x[rows] @ wu.t())
        a = ops.dequantize_mx(*ops.quantize_act_mx(a))
        out.index_add_(0, rows, ((a @ wd.t()) * wts[rows, ks][:, None]).bfloat16().float())
    return out


@pytest.mark.parametrize("M", [5, 300, 2000])
def test_moe_layer_single_rank(M):
    from quail_b200.parallel.ep import EPState
    cfg = QWEN3_MOE_GPU_TINY
    H, K, E = cfg.hidden, cfg.top_k, cfg.num_experts
    L, ex = _layer(cfg)
    st = EPState(cfg, 4096, DEV)
    ln2 = (1 + 0.1 * torch.randn(H, device=DEV)).bfloat16()
    ln1 = (1 + 0.1 * torch.randn(H, device=DEV)).bfloat16()
    for step in range(3):  # monotonic counters across layers
        h = torch.randn(M, H, device=DEV).bfloat16()
        x8, xs = ops.rmsnorm_quant_mx(h, ln2, 1e-6)
        xb = ops.rmsnorm_quant(h, ln2, 1e-6, fp8=False)
        h0 = h.float().clone()
        y8, ysf = st.forward(x8, xs, xb, h, L, next_norm=ln1)
        torch.cuda.synchronize()
        assert ops.read_and_clear_error(0) == 0
        ids = st.ids[:M * K].view(M, K).long()
        wts = st.wts[:M * K].view(M, K)
        rid, rw = ref.moe_route((xb.float() @ L["router"].float().t()).bfloat16().float(), K)
        assert (ids.sort(1).values == rid.sort(1).values).all(1).float().mean().item() > 0.9
        x = ops.dequantize_mx(x8, xs)
        want = h0 + _moe_ref(x, ids, wts, ex)
        assert rel_err(h, want) < 2e-2, (step, rel_err(h, want))
        # the expert contribution itself (h is bf16: compare against the rounded sum)
        assert rel_err(h.float() - h0, want.bfloat16().float() - h0) < 3e-2
        # the next layer's input norm
        want_n = ref.rmsnorm(h.float(), ln1.float(), 1e-6)
        assert rel_err(ops.dequantize_mx(y8, ysf), want_n) < 6e-2
        tiles, units = st.plan_header()
        cnt = torch.bincount(ids.flatten().cpu(), minlength=E)
        assert tiles == int(((cnt + 127) // 128).sum())
        assert units == int(((cnt + 31) // 32).sum())


def test_moe_pipeline_matches_fp32_model():
    from quail_b200.models.qwen3 import Qwen3Reference
    from quail_b200.models.qwen3_moe import Qwen3MoePipeline, Qwen3MoeWeights
    from quail_b200.models.weights import random_checkpoint
    from test_model_gpu import _dist, _run
    cfg = QWEN3_MOE_GPU_TINY.with_(vocab=4096, max_position=8192)
    ckpt = random_checkpoint(cfg, seed=3, device=DEV)
    ids = list(range(16))
    pipe = Qwen3MoePipeline(cfg, Qwen3MoeWeights(cfg, ckpt, DEV, head_rows=ids), max_tokens=512)
    exact = Qwen3Reference(cfg, ckpt, device=DEV, head_rows=ids)
    emul = Qwen3Reference(cfg, ckpt, device=DEV, head_rows=ids, emulate_kernels=True)
    rng = np.random.default_rng(1)
    prefix = rng.integers(0, 4096, 48).astype(np.int32)
    docs = [rng.integers(0, 4096, n).astype(np.int32) for n in (10, 200, 64, 450, 129)]
    suffix = rng.integers(0, 4096, 24).astype(np.int32)
    got = _run(pipe, cfg, prefix, docs, suffix, torch.bfloat16)
    want = _run(exact, cfg, prefix, docs, suffix, torch.float32)
    close = _run(emul, cfg, prefix, docs, suffix, torch.float32)
    assert ops.read_and_clear_error(0) == 0
    d_kernel, d_emul = _dist(got, want), _dist(close, want)
    print(f"moe: kernel-vs-exact {d_kernel:.4f} emulated-vs-exact {d_emul:.4f} kernel-vs-emulated "
          f"{_dist(got, close):.4f}")
    assert d_kernel < 1.5 * d_emul + 0.03, (d_kernel, d_emul)


def test_moe_random_weights_are_rank_independent():
    """Expert-parallel ranks build the same replicated weights from the per-layer streams."""
    from quail_b200.models.qwen3_moe import Qwen3MoeWeights
    cfg = QWEN3_MOE_GPU_TINY.with_(vocab=4096, layers=1)
    a = Qwen3MoeWeights(cfg, None, DEV, experts=range(0, 8), seed=5)
    b = Qwen3MoeWeights(cfg, None, DEV, experts=range(8, 16), seed=5)
    c = Qwen3MoeWeights(cfg, None, DEV, experts=range(0, 16), seed=5)
    assert torch.equal(a.layers[0]["wqkv"].view(torch.uint8), b.layers[0]["wqkv"].view(torch.uint8))
    assert torch.equal(a.layers[0]["router"], b.layers[0]["router"])
    half = a.layers[0]["wgu"].shape[0]
    assert torch.equal(c.layers[0]["wgu"][half:].view(torch.uint8), b.layers[0]["wgu"].view(torch.uint8))
