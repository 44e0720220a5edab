"""The Qwen3.5 vision tower: image pixels to LM token embeddings.

An image is read at a size that is a multiple of 32 pixels on each side: one
LM token per 32 x 32 pixels, made of 2 x 2 patches of 16 x 16 pixels (each
patch covers 2 frames, a still image repeats its pixels). The tower:

    x = patch_embed(patches) + interpolated learned position table
    x += proj(attention(LayerNorm(x)))     # every patch reads every patch of its image,
    x += fc2(gelu_tanh(fc1(LayerNorm(x)))) #   q and k rotated by 2-D (row, column) RoPE
    ... depth blocks ...
    tokens = fc2(gelu(fc1(LayerNorm(x) regrouped 4 patches per token)))  # the merger

Patches are ordered so that the 4 patches of one token are consecutive, token
by token, row by row (the order of the Qwen image processor). Weight names are
the checkpoints' (`model.visual.*`). `VisionReference` is the fp32 statement;
`VisionPipeline` runs the projections on the bf16 tcgen05 GEMM and the
attention on the small-tile paged attention kernel (each image one sequence
read both ways, heads padded to a built head_dim).

Reference: quail/backends/quail/executor/images.py:129-446 (pixel patches, the
encoder call through vLLM's module, image token positions); the architecture is
that of Qwen3.5 checkpoints (the Hugging Face Qwen3_5VisionModel computes the
same function, which tests/test_vision_cpu.py checks).
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from quail_b200.models.config import DecoderConfig

PREFIX = "model.visual."
PATCH_INPUT = 3 * 2 * 16 * 16     # channels x frames x patch pixels


def token_pixels(cfg: DecoderConfig) -> int:
    return cfg.vision_patch * cfg.vision_merge


def image_size(width: int, height: int, longest: int, cfg: DecoderConfig) -> tuple[int, int]:
    """(columns, rows) in LM tokens of an image read with its longer side at most `longest` pixels:
    each side rounded to whole tokens, at least one (the reference's image sizing)."""
    px = token_pixels(cfg)
    scale = min(1.0, longest / max(width, height))
    cols = max(1, round(width * scale / px))
    rows = max(1, round(height * scale / px))
    return cols, rows


def pixels(rgb: np.ndarray) -> torch.Tensor:
    """uint8 [H, W, 3] -> fp32 [3, H, W] normalized to [-1, 1] (mean 0.5, std 0.5 per channel)."""
    x = torch.from_numpy(np.array(rgb, dtype=np.uint8)).float().permute(2, 0, 1) / 255.0
    return (x - 0.5) / 0.5


def patches_of(img: torch.Tensor, cfg: DecoderConfig) -> tuple[torch.Tensor, tuple]:
    """[3, H, W] normalized pixels (H, W multiples of 32) -> ([N, 1536] patches, (1, gh, gw)):
    the 4 patches of each merged token consecutive, tokens row by row; each patch's values
    ordered (channel, frame, row, column) as the patch embedding's kernel."""
    p, m, t = cfg.vision_patch, cfg.vision_merge, cfg.vision_temporal
    C, H, W = img.shape
    gh, gw = H // p, W // p
    x = img[None].expand(t, C, H, W)                                  # a still image: the same frames
    x = x.reshape(t, C, gh // m, m, p, gw // m, m, p)
    x = x.permute(2, 5, 3, 6, 1, 0, 4, 7)                              # bh, bw, mh, mw, C, t, p, p
    return x.reshape(gh * gw, C * t * p * p).contiguous(), (1, gh, gw)


def position_table(cfg: DecoderConfig, table: torch.Tensor, gh: int, gw: int) -> torch.Tensor:
    """The learned square position table bilinearly resampled to a gh x gw patch grid, in patch
    order (merged-token blocks, as patches_of)."""
    side = int(round(math.sqrt(table.shape[0])))
    hs = torch.linspace(0, side - 1, gh, dtype=torch.float64, device=table.device)
    ws = torch.linspace(0, side - 1, gw, dtype=torch.float64, device=table.device)
    h0, w0 = hs.floor().long(), ws.floor().long()
    h1, w1 = (h0 + 1).clamp(max=side - 1), (w0 + 1).clamp(max=side - 1)
    dh, dw = (hs - h0).float(), (ws - w0).float()
    t = table.float().view(side, side, -1)

    def at(hi, wi):
        return t[hi][:, wi]                                           # [gh, gw, C]
    grid = (at(h0, w0) * ((1 - dh)[:, None, None] * (1 - dw)[None, :, None])
            + at(h0, w1) * ((1 - dh)[:, None, None] * dw[None, :, None])
            + at(h1, w0) * (dh[:, None, None] * (1 - dw)[None, :, None])
            + at(h1, w1) * (dh[:, None, None] * dw[None, :, None]))
    m = cfg.vision_merge
    C = grid.shape[-1]
    return grid.view(gh // m, m, gw // m, m, C).permute(0, 2, 1, 3, 4).reshape(gh * gw, C)


def rotary_2d(cfg: DecoderConfig, gh: int, gw: int, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) [N, head_dim] of each patch: the first quarter-frequencies rotate by the patch's
    row, the next by its column (rotate-half pairs over the whole head)."""
    hd = cfg.vision_hidden // cfg.vision_heads
    quarter = hd // 4
    inv = 1.0 / (10000.0 ** (torch.arange(0, hd // 2, 2, dtype=torch.float32, device=device) / (hd // 2)))
    m = cfg.vision_merge
    r = torch.arange(gh, device=device).view(gh // m, m)[:, None, :, None].expand(gh // m, gw // m, m, m)
    c = torch.arange(gw, device=device).view(gw // m, m)[None, :, None, :].expand(gh // m, gw // m, m, m)
    r, c = r.reshape(-1).float(), c.reshape(-1).float()
    ang = torch.cat([r[:, None] * inv[None, :quarter], c[:, None] * inv[None, :quarter]], dim=1)
    emb = torch.cat([ang, ang], dim=1)
    return emb.cos(), emb.sin()


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [N, heads, d] rotated pairwise (i, i + d/2)."""
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


def random_vision(cfg: DecoderConfig, gen: torch.Generator, device="cpu", dtype=torch.bfloat16) -> dict:
    """Random-init vision tower tensors in checkpoint names (LayerNorms at one / zero)."""
    Hd, I, out = cfg.vision_hidden, cfg.vision_intermediate, cfg.hidden
    p, t = cfg.vision_patch, cfg.vision_temporal

    def r(*shape, std=0.02):
        return (torch.randn(*shape, generator=gen, device=device) * std).to(dtype)

    w = {PREFIX + "patch_embed.proj.weight": r(Hd, 3, t, p, p), PREFIX + "patch_embed.proj.bias": r(Hd),
         PREFIX + "pos_embed.weight": r(cfg.vision_pos_embeddings, Hd)}
    for i in range(cfg.vision_depth):
        b = f"{PREFIX}blocks.{i}."
        for n in ("norm1", "norm2"):
            w[b + n + ".weight"] = torch.ones(Hd, device=device, dtype=dtype)
            w[b + n + ".bias"] = torch.zeros(Hd, device=device, dtype=dtype)
        w.update({b + "attn.qkv.weight": r(3 * Hd, Hd), b + "attn.qkv.bias": r(3 * Hd),
                  b + "attn.proj.weight": r(Hd, Hd), b + "attn.proj.bias": r(Hd),
                  b + "mlp.linear_fc1.weight": r(I, Hd), b + "mlp.linear_fc1.bias": r(I),
                  b + "mlp.linear_fc2.weight": r(Hd, I), b + "mlp.linear_fc2.bias": r(Hd)})
    M = Hd * cfg.vision_merge ** 2
    w.update({PREFIX + "merger.norm.weight": torch.ones(Hd, device=device, dtype=dtype),
              PREFIX + "merger.norm.bias": torch.zeros(Hd, device=device, dtype=dtype),
              PREFIX + "merger.linear_fc1.weight": r(M, M), PREFIX + "merger.linear_fc1.bias": r(M),
              PREFIX + "merger.linear_fc2.weight": r(out, M), PREFIX + "merger.linear_fc2.bias": r(out)})
    return w


class VisionReference:
    """fp32 forward of the vision tower (CPU or GPU)."""

    def __init__(self, cfg: DecoderConfig, ckpt: dict, device="cpu"):
        assert cfg.has_vision
        self.cfg = cfg
        self.device = device
        self.w = {k[len(PREFIX):]: v.to(device=device, dtype=torch.float32) for k, v in ckpt.items()
                  if k.startswith(PREFIX)}

    @torch.no_grad()
    def encode(self, images: list[torch.Tensor]) -> list[torch.Tensor]:
        """Normalized [3, H, W] images -> per image its token embeddings [H*W/1024, LM hidden] (fp32)."""
        return [self._one(img) for img in images]

    def _one(self, img: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        Hd, nh = cfg.vision_hidden, cfg.vision_heads
        patches, (_, gh, gw) = patches_of(img.to(self.device), cfg)
        x = patches @ w["patch_embed.proj.weight"].reshape(Hd, -1).t() + w["patch_embed.proj.bias"]
        x = x + position_table(cfg, w["pos_embed.weight"], gh, gw).to(x.device)
        cos, sin = rotary_2d(cfg, gh, gw, device=x.device)
        n = x.shape[0]
        for i in range(cfg.vision_depth):
            b = f"blocks.{i}."
            y = F.layer_norm(x, (Hd,), w[b + "norm1.weight"], w[b + "norm1.bias"], 1e-6)
            qkv = (y @ w[b + "attn.qkv.weight"].t() + w[b + "attn.qkv.bias"]).view(n, 3, nh, Hd // nh)
            q, k, v = _rotate(qkv[:, 0], cos, sin), _rotate(qkv[:, 1], cos, sin), qkv[:, 2]
            s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(Hd // nh)
            o = torch.einsum("hqk,khd->qhd", s.softmax(-1), v).reshape(n, Hd)
            x = x + o @ w[b + "attn.proj.weight"].t() + w[b + "attn.proj.bias"]
            y = F.layer_norm(x, (Hd,), w[b + "norm2.weight"], w[b + "norm2.bias"], 1e-6)
            y = gelu_tanh(y @ w[b + "mlp.linear_fc1.weight"].t() + w[b + "mlp.linear_fc1.bias"])
            x = x + y @ w[b + "mlp.linear_fc2.weight"].t() + w[b + "mlp.linear_fc2.bias"]
        y = F.layer_norm(x, (Hd,), w["merger.norm.weight"], w["merger.norm.bias"], 1e-6)
        y = y.reshape(n // cfg.vision_merge ** 2, -1)
        y = F.gelu(y @ w["merger.linear_fc1.weight"].t() + w["merger.linear_fc1.bias"])
        return y @ w["merger.linear_fc2.weight"].t() + w["merger.linear_fc2.bias"]


class VisionPipeline:
    """The vision tower on the GPU: projections on the bf16 tcgen05 GEMM, attention on the
    small-tile paged attention kernel (each image one sequence read both ways; heads padded
    with zeros to a head_dim the kernel is built for, which leaves the dot products and the
    first head_dim outputs unchanged); norms, biases and activations in PyTorch."""

    PAGE = 16

    def __init__(self, cfg: DecoderConfig, ckpt: dict, device):
        assert cfg.has_vision
        self.cfg = cfg
        self.device = torch.device(device)
        bf = torch.bfloat16
        w = {k[len(PREFIX):]: v.to(device=device) for k, v in ckpt.items() if k.startswith(PREFIX)}
        self.w = {k: (v.to(bf).contiguous() if v.dim() == 2 else v.float()) for k, v in w.items()}
        self.w["patch_embed.proj.weight"] = w["patch_embed.proj.weight"].reshape(cfg.vision_hidden, -1).to(bf) \
            .contiguous()
        # the GEMM reads K in 128-column blocks: the MLP width is padded with zero units
        I = cfg.vision_intermediate
        pad = -I % 128
        if pad:
            for i in range(cfg.vision_depth):
                b = f"blocks.{i}.mlp."
                self.w[b + "linear_fc1.weight"] = F.pad(self.w[b + "linear_fc1.weight"], (0, 0, 0, pad)).contiguous()
                self.w[b + "linear_fc1.bias"] = F.pad(self.w[b + "linear_fc1.bias"], (0, pad))
                self.w[b + "linear_fc2.weight"] = F.pad(self.w[b + "linear_fc2.weight"], (0, pad)).contiguous()
        self.hd = cfg.vision_hidden // cfg.vision_heads
        self.pad = 64 if self.hd <= 64 else (128 if self.hd <= 128 else 256)

    def _lin(self, x: torch.Tensor, name: str) -> torch.Tensor:
        from quail_b200 import ops
        return ops.gemm(x.to(torch.bfloat16).contiguous(), self.w[name + ".weight"]).float() + self.w[name + ".bias"]

    @torch.no_grad()
    def encode(self, images: list[torch.Tensor]) -> list[torch.Tensor]:
        from quail_b200 import ops
        cfg, w = self.cfg, self.w
        Hd, nh, hd, D = cfg.vision_hidden, cfg.vision_heads, self.hd, self.pad
        dev = self.device
        parts, grids = [], []
        for img in images:
            p, (_, gh, gw) = patches_of(img.to(dev), cfg)
            parts.append(p)
            grids.append((gh, gw))
        x = self._lin(torch.cat(parts), "patch_embed.proj")
        x = x + torch.cat([position_table(cfg, w["pos_embed.weight"].float(), gh, gw).to(dev) for gh, gw in grids])
        cs = [rotary_2d(cfg, gh, gw, device=dev) for gh, gw in grids]
        cos, sin = torch.cat([c for c, _ in cs]), torch.cat([s_ for _, s_ in cs])
        n = x.shape[0]
        # each image one sequence over its own scratch pages, read both ways
        P = self.PAGE
        rows, seqs, page = 0, [], 0
        for gh, gw in grids:
            L = gh * gw
            seqs.append([rows, L, 1, 1, L, 0, 0, 0, page, 0, 0, 0])
            rows += L
            page += -(-L // P)
        seqs_t = torch.tensor(seqs, dtype=torch.int32)
        tiles = _tiles(seqs_t).to(dev)
        seqs_d = seqs_t.to(dev)
        slots = []
        for (gh, gw), sq in zip(grids, seqs):
            slots.append(sq[8] * P + torch.arange(gh * gw))
        slots = torch.cat(slots).to(dev).long()
        page_list = torch.arange(page, dtype=torch.int32, device=dev)
        kc = torch.zeros(page, P, nh, D, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        no_decode = torch.zeros(0, dtype=torch.int32, device=dev)
        for i in range(cfg.vision_depth):
            b = f"blocks.{i}."
            y = F.layer_norm(x, (Hd,), w[b + "norm1.weight"], w[b + "norm1.bias"], 1e-6)
            qkv = self._lin(y, b + "attn.qkv").view(n, 3, nh, hd)
            q, k = _rotate(qkv[:, 0], cos, sin), _rotate(qkv[:, 1], cos, sin)
            qp = torch.zeros(n, nh, D, dtype=torch.bfloat16, device=dev)
            qp[..., :hd] = q
            kc.view(-1, nh, D)[slots, :, :hd] = k.to(torch.bfloat16)
            vc.view(-1, nh, D)[slots, :, :hd] = qkv[:, 2].to(torch.bfloat16)
            o = torch.empty(n, nh * D, dtype=torch.bfloat16, device=dev)
            ops.small_attention(qp, kc, vc, seqs_d, tiles, no_decode, page_list, 1.0 / math.sqrt(hd), o)
            o = o.view(n, nh, D)[..., :hd].reshape(n, Hd)
            x = x + self._lin(o, b + "attn.proj")
            y = F.layer_norm(x, (Hd,), w[b + "norm2.weight"], w[b + "norm2.bias"], 1e-6)
            x = x + self._lin(gelu_tanh(self._lin(y, b + "mlp.linear_fc1")), b + "mlp.linear_fc2")
        y = F.layer_norm(x, (Hd,), w["merger.norm.weight"], w["merger.norm.bias"], 1e-6)
        y = y.reshape(n // cfg.vision_merge ** 2, -1)
        y = self._lin(F.gelu(self._lin(y, "merger.linear_fc1")), "merger.linear_fc2")
        counts = [gh * gw // cfg.vision_merge ** 2 for gh, gw in grids]
        return list(y.split(counts))


def _tiles(seqs: torch.Tensor) -> torch.Tensor:
    from quail_b200.ops import reference as ref
    return ref.attention_tiles(seqs)
