"""fp8 (e4m3) block quantization in the checkpoint and kernel layouts.

Weights: HF `weight_scale_inv` layout, one fp32 scale per 128x128 block,
[ceil(N/128), K/128] (Qwen/Qwen3-*-FP8 checkpoints; reference spec
quail/specs/data/models/qwen3-4b-fp8.toml). Activations: one fp32 scale per
token and 128-wide K group, stored transposed [K/128, T] so that one K
block's scales are contiguous over tokens (the "column-major scales" of the
reference's per_token_group_fp8_quant call, attention.py:517-532).
"""

from __future__ import annotations

import torch

FP8_MAX = 448.0


def quantize_weight(w: torch.Tensor, block: int = 128):
    """[N, K] float -> (e4m3 [N, K], fp32 scales [ceil(N/block), K/block]) by block amax."""
    N, K = w.shape
    assert K % 128 == 0
    nb = (N + block - 1) // block
    wp = torch.zeros(nb * block, K, dtype=torch.float32, device=w.device)
    wp[:N] = w.float()
    blocks = wp.view(nb, block, K // 128, 128)
    amax = blocks.abs().amax(dim=(1, 3)).clamp(min=1e-12)
    scale = amax / FP8_MAX
    q = (blocks / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX)
    q = q.view(nb * block, K)[:N].to(torch.float8_e4m3fn)
    return q.contiguous(), scale.contiguous()


def dequantize_weight(q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    N, K = q.shape
    s = scale.repeat_interleave(block, dim=0)[:N].repeat_interleave(128, dim=1)
    return q.float() * s


def quantize_act(x: torch.Tensor):
    """[T, K] float -> (e4m3 [T, K], scales [K/128, T]) with one scale per 128 columns."""
    T, K = x.shape
    g = x.float().view(T, K // 128, 128)
    amax = g.abs().amax(dim=2).clamp(min=1e-12)
    scale = amax / FP8_MAX
    q = (g / scale[:, :, None]).clamp(-FP8_MAX, FP8_MAX).view(T, K).to(torch.float8_e4m3fn)
    return q, scale.t().contiguous()


def dequantize_act(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    T, K = q.shape
    s = scale[:, :T].t().repeat_interleave(128, dim=1)
    return q.float() * s


def interleave_gate_up(w: torch.Tensor, scale: torch.Tensor | None = None, block: int = 128):
    """Reorder a [2I, K] gate_up weight for the fused SwiGLU epilogue.

    Each 256-row tile t holds [gate 128t..+63 | up 128t..+63 | gate 128t+64..+127 |
    up 128t+64..+127]. With scales (e4m3 weights), the 128x128 block scales
    are expanded to one scale per 64 rows of the new order.
    """
    I2, K = w.shape
    inter = I2 // 2
    assert inter % 128 == 0
    gate = w[:inter].view(inter // 64, 64, K)
    up = w[inter:].view(inter // 64, 64, K)
    # groups of 64 rows: g0 u0 g1 u1 ...
    out = torch.stack([gate, up], dim=1).reshape(I2, K)
    if scale is None:
        return out.contiguous()
    # original row of each 64-row group of the new order
    groups = torch.arange(I2 // 64, device=w.device)
    src_group = torch.where(groups % 2 == 0, groups // 2, inter // 64 + groups // 2)
    src_block = (src_group * 64) // block
    return out.contiguous(), scale[src_block].contiguous()
