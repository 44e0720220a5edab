"""LFM3 (d1) set-attention passes on the kernels against the fp32 statement."""

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


@pytest.mark.parametrize("win", [16, 64, 256])
def test_sliding_window_in_the_small_tile_kernel(win):
    from test_kernels_gpu import _segmented_case
    specs = [(300, [300]), (70, [70]), (40, [200, 40]), (1, [1]), (129, [129])]
    QH, KH, D = 8, 2, 128
    q, kc, vc, seqs, pl = _segmented_case(16, specs, QH=QH, KH=KH, D=D, pages=2048)
    seqs[:, 3] = win << 8
    scale = ref.softmax_scale(D)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale)
    T = q.shape[0]
    out = torch.empty(T, QH * D, dtype=torch.bfloat16, device=DEV)
    ops.small_attention(q, kc, vc, seqs.to(DEV), ref.attention_tiles(seqs).to(DEV),
                        torch.zeros(0, dtype=torch.int32, device=DEV), pl.to(DEV), scale, out)
    assert rel_err(out.view(T, QH, D), want.view(T, QH, D)) < 1e-2


def test_sandwich_norm_and_kv_row_copy():
    T, H = 300, 1024
    y = torch.randn(T, H, device=DEV).bfloat16()
    h = torch.randn(T, H, device=DEV).bfloat16()
    w1 = (1 + 0.2 * torch.randn(H, device=DEV)).bfloat16()
    w2 = (1 + 0.2 * torch.randn(H, device=DEV)).bfloat16()
    h0 = h.float().clone()
    x = ops.post_norm_add_norm(y, h, w1, w2, 1e-5)
    want_h = h0 + ref.rmsnorm(y.float(), w1.float(), 1e-5)
    assert rel_err(h, want_h) < 1e-2
    assert rel_err(x, ref.rmsnorm(want_h, w2.float(), 1e-5)) < 1e-2
    kc = torch.randn(8, 16, 2, 128, device=DEV).bfloat16()
    vc = torch.randn_like(kc)
    src = torch.tensor([3, 17, 40], dtype=torch.int32, device=DEV)
    dst = torch.tensor([100, 101, 5], dtype=torch.int32, device=DEV)
    k0, v0 = kc.view(-1, 2, 128).clone(), vc.view(-1, 2, 128).clone()
    ops.kv_copy_rows(kc, vc, src, dst)
    assert torch.equal(kc.view(-1, 2, 128)[dst.long()], k0[src.long()])
    assert torch.equal(vc.view(-1, 2, 128)[dst.long()], v0[src.long()])


def test_set_passes_on_the_kernels_match_the_fp32_model():
    from quail_b200.models.build import random_checkpoint_on
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.models.lfm3 import Lfm3Pipeline, Lfm3Reference, SetPass
    cfg = MODEL_CONFIGS["d1-gpu-tiny"]
    ckpt = random_checkpoint_on(cfg, DEV, seed=4)
    pipe = Lfm3Pipeline(cfg, ckpt, DEV, max_tokens=4096)
    exact = Lfm3Reference(cfg, ckpt, device=DEV)
    rng = np.random.default_rng(2)
    passes = []
    for state, qlens in ((40, [9, 12, 7]), (150, [20]), (300, [8, 8, 8, 8]), (17, [30, 5])):
        toks = rng.integers(0, cfg.vocab, state + sum(qlens)).astype(np.int32)
        ends, row = [], state
        for n in qlens:
            row += n
            ends.append(row - 1)
        passes.append(SetPass(toks, state, qlens, ends + [state - 1, 3]))
    got = pipe.forward_passes(passes)
    want = exact.forward_passes(passes)
    for g, w in zip(got, want):
        assert rel_err(g, w) < 0.05, rel_err(g, w)
