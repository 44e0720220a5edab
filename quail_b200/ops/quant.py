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


# ---------------------------------------------------------------- MX (UE8M0) formats
#
# The tcgen05 block-scaled MMA (kind::mxf8f6f4.block_scale) takes one
# power-of-two scale byte (UE8M0: value 2^(e - 127)) per row and 32-wide K
# block. The kernels read them in the scale-factor atom layout: per
# 128-row x 128-K chunk, 512 bytes with row r, K block j at byte
# (r % 32) * 16 + ((r % 128) // 32) * 4 + j; chunks ordered [row/128][K/128].

def ue8m0_exponent(amax: torch.Tensor) -> torch.Tensor:
    """Biased exponent of the smallest power of two >= amax / 448 (clamped to [1, 253])."""
    s = (amax.float().clamp(min=1e-30) / FP8_MAX)
    bits = s.view(torch.int32)
    e = (bits >> 23) & 0xFF
    e = e + ((bits & 0x7FFFFF) != 0).to(torch.int32)
    return e.clamp(1, 253).to(torch.uint8)


def ue8m0_value(e: torch.Tensor) -> torch.Tensor:
    return torch.exp2(e.float() - 127.0)


def pack_sf_atoms(e: torch.Tensor) -> torch.Tensor:
    """[R, K/32] uint8 exponents -> flat uint8 in the atom layout."""
    R, KB = e.shape
    assert KB % 4 == 0
    Rp = -(-R // 128) * 128
    ep = torch.zeros(Rp, KB, dtype=torch.uint8, device=e.device)
    ep[:R] = e
    x = ep.view(Rp // 128, 4, 32, KB // 4, 4).permute(0, 3, 2, 1, 4)
    return x.contiguous().view(-1)


def unpack_sf_atoms(sf: torch.Tensor, R: int, K: int) -> torch.Tensor:
    """Inverse of pack_sf_atoms -> [R, K/32] uint8."""
    KB = K // 32
    Rp = -(-R // 128) * 128
    x = sf[:(Rp // 128) * (KB // 4) * 512].view(Rp // 128, KB // 4, 32, 4, 4).permute(0, 3, 2, 1, 4)
    return x.contiguous().view(Rp, KB)[:R]


def quantize_act_mx(x: torch.Tensor, group: int = 32):
    """[T, K] float -> (e4m3 [T, K], atom-packed UE8M0 bytes), one scale per `group` columns."""
    T, K = x.shape
    g = x.float().view(T, K // group, group)
    e = ue8m0_exponent(g.abs().amax(dim=2))
    q = (g / ue8m0_value(e)[:, :, None]).clamp(-FP8_MAX, FP8_MAX).view(T, K).to(torch.float8_e4m3fn)
    e32 = e.repeat_interleave(group // 32, dim=1)
    return q, pack_sf_atoms(e32)


def quantize_weight_mx(w: torch.Tensor, block: int = 128):
    """[N, K] float -> (e4m3 [N, K], atom-packed UE8M0 bytes) with power-of-two 128x128 block scales."""
    N, K = w.shape
    nb = -(-N // block)
    wp = torch.zeros(nb * block, K, dtype=torch.float32, device=w.device)
    wp[:N] = w.float()
    blocks = wp.view(nb, block, K // 128, 128)
    e = ue8m0_exponent(blocks.abs().amax(dim=(1, 3)))          # [nb, K/128]
    q = (blocks / ue8m0_value(e)[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX)
    q = q.view(nb * block, K)[:N].to(torch.float8_e4m3fn)
    rows = e.repeat_interleave(block, dim=0)[:N].repeat_interleave(4, dim=1)  # [N, K/32]
    return q.contiguous(), pack_sf_atoms(rows)


def requantize_weight_mx(q: torch.Tensor, scale: torch.Tensor, block: int = 128):
    """HF fp8 weight + fp32 128x128 `weight_scale_inv` -> the MX (power-of-two scale) form."""
    return quantize_weight_mx(dequantize_weight(q, scale, block), block)


def dequantize_mx(q: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    R, K = q.shape
    e = unpack_sf_atoms(sf, R, K)
    return q.float() * ue8m0_value(e).repeat_interleave(32, dim=1)


def interleave_gate_up_mx(w: torch.Tensor, block: int = 128):
    """fp32/bf16 [2I, K] gate_up -> MX-quantized, rows interleaved for the SwiGLU epilogue.

    Quantizes gate and up separately with 128x128 blocks, then reorders the
    rows (64-row groups g0 u0 g1 u1 ...) together with their scale rows.
    """
    I2, K = w.shape
    inter = I2 // 2
    qg, sg = quantize_weight_mx(w[:inter], block)
    qu, su = quantize_weight_mx(w[inter:], block)
    eg, eu = unpack_sf_atoms(sg, inter, K), unpack_sf_atoms(su, inter, K)
    q = torch.stack([qg.view(inter // 64, 64, K), qu.view(inter // 64, 64, K)], dim=1).reshape(I2, K)
    e = torch.stack([eg.view(inter // 64, 64, -1), eu.view(inter // 64, 64, -1)], dim=1).reshape(I2, -1)
    return q.contiguous(), pack_sf_atoms(e)


# ---------------------------------------------------------------- NVFP4
# E2M1 values by code (sign in bit 3): 0, 0.5, 1, 1.5, 2, 3, 4, 6
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
FP4_MAX = 6.0


def _e2m1_codes(x: torch.Tensor) -> torch.Tensor:
    """Round to the nearest E2M1 value (ties to the even code); 4-bit codes as uint8."""
    grid = torch.tensor(E2M1_VALUES, device=x.device)
    a = x.abs().clamp(max=FP4_MAX)
    d = (a[..., None] - grid).abs()
    best = d.min(dim=-1, keepdim=True).values
    # among equally near values the even code (codes 0..7 in order of value)
    cand = torch.where(d <= best + 1e-12, torch.arange(8, device=x.device), 99)
    even = torch.where(cand % 2 == 0, cand, 99).min(dim=-1).values
    code = torch.where(even < 99, even, cand.min(dim=-1).values)
    return (code | ((x < 0) & (code > 0)).to(code.dtype) * 8).to(torch.uint8)


def quantize_nvfp4(x: torch.Tensor, global_scale: float | None = None):
    """[R, K] float -> (packed E2M1 [R, K/2] uint8, UE4M3 block-scale atoms, global scale).

    One e4m3 scale per row and 16 values (amax / 6, divided by the global
    scale so that it fits e4m3's range: global = amax(x) / (448 * 6)); two
    codes per byte, the even element in the low nibble. Dequantized value =
    E2M1 x block scale x global scale.
    """
    R, K = x.shape
    assert K % 64 == 0
    xf = x.float()
    if global_scale is None:
        global_scale = max(float(xf.abs().max()), 1e-12) / (FP8_MAX * FP4_MAX)
    g = xf.view(R, K // 16, 16)
    bs = (g.abs().amax(dim=2) / FP4_MAX / global_scale).clamp(max=FP8_MAX)
    bs8 = bs.to(torch.float8_e4m3fn)
    scale = bs8.float() * global_scale
    q = torch.where(scale[..., None] > 0, g / scale[..., None].clamp(min=1e-30), torch.zeros_like(g))
    codes = _e2m1_codes(q).view(R, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    return packed, pack_sf_atoms(bs8.view(torch.uint8)), global_scale


def dequantize_nvfp4(packed: torch.Tensor, sf: torch.Tensor, global_scale: float, K: int) -> torch.Tensor:
    """Inverse of quantize_nvfp4 -> fp32 [R, K]."""
    R = packed.shape[0]
    lo, hi = packed & 0xF, packed >> 4
    codes = torch.stack([lo, hi], dim=-1).view(R, K).long()
    vals = torch.tensor(E2M1_VALUES, device=packed.device)[codes & 7] * torch.where(codes >= 8, -1.0, 1.0)
    KB = K // 16
    Rp = -(-R // 128) * 128
    e = sf[:(Rp // 128) * (KB // 4) * 512].view(Rp // 128, KB // 4, 32, 4, 4).permute(0, 3, 2, 1, 4)
    bs = e.contiguous().view(Rp, KB)[:R].view(torch.float8_e4m3fn).float()
    return vals * bs.repeat_interleave(16, dim=1) * global_scale


def fake_nvfp4_rows(x: torch.Tensor) -> torch.Tensor:
    """fp32 values of the per-row dynamic NVFP4 quantization of x [R, K] (the GPU quantizer's
    rule: row scale amax / (448 * 6), e4m3 block scales of 16 values, E2M1 codes)."""
    R, K = x.shape
    xf = x.float()
    g = (xf.abs().amax(dim=1, keepdim=True).clamp(min=1e-30) / (FP8_MAX * FP4_MAX))      # [R, 1]
    blocks = xf.view(R, K // 16, 16)
    bs = (blocks.abs().amax(dim=2) / FP4_MAX / g).to(torch.float8_e4m3fn).float()         # [R, K/16]
    scale = bs * g
    q = torch.where(scale[..., None] > 0, blocks / scale[..., None].clamp(min=1e-30), torch.zeros_like(blocks))
    codes = _e2m1_codes(q).long()
    vals = torch.tensor(E2M1_VALUES, device=x.device)[codes & 7] * torch.where(codes >= 8, -1.0, 1.0)
    return (vals * scale[..., None]).view(R, K)
