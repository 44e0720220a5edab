"""LFM2 hybrid decoder: gated short convolutions and GQA attention.

Every layer is `h += mixer(RMSNorm(h)); h += SwiGLU(RMSNorm(h))` (operator_norm,
ffn_norm), the final norm is `embedding_norm`, the head is tied. Mixers:

  conv  B, C, x = in_proj(h);  y = C * causal_depthwise_conv(B * x)  (width 3,
        no bias, no activation);  out_proj(y). The window (last two values of
        B * x per channel) lives in the key's arena state slot, like the Gated
        DeltaNet state of Qwen3.5: a sequence continues its own slot or starts
        from the slot of the last segment it reads.
  attn  q/k/v projections, per-head RMSNorm of q and k, full NeoX RoPE, paged
        GQA attention (head_dim 64), out_proj.

`Lfm2Reference` is the fp32 PyTorch statement (CPU or GPU); `Lfm2Pipeline`
runs the sm_100a kernels (bf16 tcgen05 GEMMs, the short_conv kernel, the q/k
norm + RoPE + KV write and small-tile attention kernels).

Reference: quail/backends/quail/executor/models/lfm2.py (the reference's
LFM2 pipeline over vLLM modules); HF names of LiquidAI/LFM2 checkpoints.
"""

from __future__ import annotations

import torch

from quail_b200.models.config import DecoderConfig
from quail_b200.models.weights import dequantized, final_norm_name, head_weight
from quail_b200.ops import reference as ref


def short_conv_ref(bcx: torch.Tensor, window: torch.Tensor, w: torch.Tensor):
    """bcx [n, 3H] -> (C * conv(B * x) [n, H], new window [W-1, H]); w [H, W]."""
    H = w.shape[0]
    B, C, x = bcx[:, :H].float(), bcx[:, H:2 * H].float(), bcx[:, 2 * H:].float()
    bx = B * x
    full = torch.cat([window.float(), bx], dim=0)
    n, width = bx.shape[0], w.shape[1]
    acc = torch.zeros_like(bx)
    for j in range(width):
        acc += full[j:j + n] * w[:, j].float()
    return C * acc, full[-(width - 1):].clone()


class Lfm2Reference:
    """fp32 forward over packed chunks (same contract as Qwen3Reference)."""

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor], device="cpu", head_rows=None,
                 dtype=torch.float32):
        assert cfg.arch == "lfm2"
        self.cfg = cfg
        self.device = device
        f = lambda t: t.to(device=device, dtype=dtype)  # noqa: E731
        self.embed = f(ckpt["model.embed_tokens.weight"])
        self.final_norm = f(ckpt[final_norm_name(cfg)])
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            L = {"ln1": f(ckpt[p + "operator_norm.weight"]), "ln2": f(ckpt[p + "ffn_norm.weight"]),
                 "wg": f(dequantized(ckpt, p + "feed_forward.w1")), "wu": f(dequantized(ckpt, p + "feed_forward.w3")),
                 "wd": f(dequantized(ckpt, p + "feed_forward.w2"))}
            if cfg.kind(i) == "conv":
                L.update(win=f(dequantized(ckpt, p + "conv.in_proj")), wout=f(dequantized(ckpt, p + "conv.out_proj")),
                         conv=f(ckpt[p + "conv.conv.weight"][:, 0, :]))
            else:
                q = p + "self_attn."
                L.update(wq=f(dequantized(ckpt, q + "q_proj")), wk=f(dequantized(ckpt, q + "k_proj")),
                         wv=f(dequantized(ckpt, q + "v_proj")), wo=f(dequantized(ckpt, q + "out_proj")),
                         qn=f(ckpt[q + "q_layernorm.weight"]), kn=f(ckpt[q + "k_layernorm.weight"]))
            self.layers.append(L)
        self.head = f(head_weight(ckpt, cfg))
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.head_dim, cfg.rope_theta, device=device)
        self.scale = ref.softmax_scale(cfg.head_dim)
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def set_answer_rows(self, token_ids) -> None:
        ids = torch.as_tensor(list(token_ids), dtype=torch.long, device=self.head.device)
        self.answer_rows = self.head.index_select(0, ids)
        self.answer_ids = ids.cpu()

    @torch.no_grad()
    def hidden_chunk(self, chunk, arena) -> torch.Tensor:
        cfg = self.cfg
        QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        h = self.embed[chunk.ids.long()]
        T = h.shape[0]
        state = arena.states["sconv"]
        seqs = chunk.seqs.cpu()
        sio = chunk.state_io.cpu()
        ci = ai = 0
        for i, L in enumerate(self.layers):
            x = ref.rmsnorm(h, L["ln1"], cfg.rms_eps)
            if cfg.kind(i) == "conv":
                bcx = x @ L["win"].t()
                y = torch.empty(T, cfg.hidden, dtype=h.dtype, device=h.device)
                for s in range(seqs.shape[0]):
                    q0, n = int(seqs[s, 0]), int(seqs[s, 1])
                    src, dst = int(sio[s, 0]), int(sio[s, 1])
                    win = state[src, ci].clone() if src >= 0 else torch.zeros_like(state[0, ci])
                    out, win = short_conv_ref(bcx[q0:q0 + n], win, L["conv"])
                    state[dst, ci] = win
                    y[q0:q0 + n] = out.to(y.dtype)
                h = h + y @ L["wout"].t()
                ci += 1
            else:
                kc, vc = arena.layer(ai)
                q = ref.rope_neox(ref.rmsnorm((x @ L["wq"].t()).view(T, QH, D), L["qn"], cfg.rms_eps),
                                  chunk.positions, self.cos_sin)
                k = ref.rope_neox(ref.rmsnorm((x @ L["wk"].t()).view(T, KH, D), L["kn"], cfg.rms_eps),
                                  chunk.positions, self.cos_sin)
                v = (x @ L["wv"].t()).view(T, KH, D)
                ok = chunk.slots >= 0
                slots = chunk.slots[ok].long()
                kc.view(-1, KH, D)[slots] = k[ok].to(kc.dtype)
                vc.view(-1, KH, D)[slots] = v[ok].to(vc.dtype)
                o = ref.segmented_attention(q, kc, vc, chunk.seqs, chunk.page_list, self.scale).to(h.dtype)
                h = h + o @ L["wo"].t()
                ai += 1
            x = ref.rmsnorm(h, L["ln2"], cfg.rms_eps)
            h = h + ref.silu_mul(x @ L["wg"].t(), x @ L["wu"].t()) @ L["wd"].t()
        return h

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        h = self.hidden_chunk(chunk, arena)
        normed = ref.rmsnorm(h[chunk.final_rows.long()], self.final_norm, self.cfg.rms_eps)
        ans = (normed @ self.answer_rows.t()).float()
        if not getattr(chunk, "full_readout", False):
            return ans
        full = (normed @ self.head.t()).float()
        return ref.head_readout(full, ans, getattr(chunk, "topk", False))


class Lfm2Pipeline:
    """Forward pass of a packed chunk of an LFM2 model on the GPU kernels (bf16 weights)."""

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor], device, head_rows=None):
        from quail_b200.ops.quant import interleave_gate_up
        assert cfg.arch == "lfm2" and cfg.head_dim in (64, 128, 256)
        self.cfg = cfg
        self.device = device
        bf = torch.bfloat16

        def proj(name):
            return dequantized(ckpt, name).to(device=device, dtype=bf).contiguous()

        self.embed = ckpt["model.embed_tokens.weight"].to(device=device, dtype=bf).contiguous()
        self.final_norm = ckpt[final_norm_name(cfg)].to(device=device, dtype=bf)
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            L = {"ln1": ckpt[p + "operator_norm.weight"].to(device=device, dtype=bf),
                 "ln2": ckpt[p + "ffn_norm.weight"].to(device=device, dtype=bf),
                 "wgu": interleave_gate_up(torch.cat([proj(p + "feed_forward.w1"), proj(p + "feed_forward.w3")])),
                 "wd": proj(p + "feed_forward.w2")}
            if cfg.kind(i) == "conv":
                L.update(win=proj(p + "conv.in_proj"), wout=proj(p + "conv.out_proj"),
                         conv=ckpt[p + "conv.conv.weight"][:, 0, :].to(device=device, dtype=torch.float32)
                         .contiguous())
            else:
                q = p + "self_attn."
                L.update(wqkv=torch.cat([proj(q + "q_proj"), proj(q + "k_proj"), proj(q + "v_proj")]).contiguous(),
                         wo=proj(q + "out_proj"),
                         qn=ckpt[q + "q_layernorm.weight"].to(device=device, dtype=bf).contiguous(),
                         kn=ckpt[q + "k_layernorm.weight"].to(device=device, dtype=bf).contiguous())
            self.layers.append(L)
        self.head = head_weight(ckpt, cfg)
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.head_dim, cfg.rope_theta, device=device)
        self.scale = ref.softmax_scale(cfg.head_dim)
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def set_answer_rows(self, token_ids) -> None:
        ids = torch.as_tensor(list(token_ids), dtype=torch.long)
        self.answer_rows = self.head.index_select(0, ids.to(self.head.device)).to(
            device=self.device, dtype=torch.bfloat16).contiguous()
        self.answer_ids = ids

    def head_bf16(self) -> torch.Tensor:
        if getattr(self, "_head_dev", None) is None:
            self._head_dev = self.head.to(device=self.device, dtype=torch.bfloat16).contiguous()
        return self._head_dev

    @torch.no_grad()
    def forward_hidden(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        C = ops.native()
        cfg = self.cfg
        T = chunk.num_tokens
        QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        h = ops.embed_gather(chunk.ids, self.embed)
        ci = ai = 0
        for i, L in enumerate(self.layers):
            x = ops.rmsnorm_quant(h, L["ln1"], cfg.rms_eps, fp8=False)
            if cfg.kind(i) == "conv":
                bcx = ops.gemm(x, L["win"])
                y = torch.empty(T, cfg.hidden, dtype=torch.bfloat16, device=self.device)
                ops.count_launch()
                C.short_conv(bcx, L["conv"], chunk.seqs, chunk.state_io, arena.states["sconv"], ci, y)
                ops.gemm(y, L["wout"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
                ci += 1
            else:
                p = ops.gemm(x, L["wqkv"])
                kc, vc = arena.layer(ai)
                q = torch.empty(T, QH, D, dtype=torch.bfloat16, device=self.device)
                ops.count_launch(1)
                C.hybrid_qk_rope_kv(p, QH, KH, False, chunk.positions, L["qn"], L["kn"], False, self.cos_sin,
                                    chunk.slots, kc, vc, q, cfg.rms_eps, 0, 0)
                o = torch.empty(T, QH * D, dtype=torch.bfloat16, device=self.device)
                ops.small_attention(q, kc, vc, chunk.seqs, chunk.tiles, chunk.dseqs, chunk.page_list, self.scale, o,
                                  None, 0)
                ops.gemm(o, L["wo"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
                ai += 1
            x = ops.rmsnorm_quant(h, L["ln2"], cfg.rms_eps, fp8=False)
            a = ops.gemm(x, L["wgu"], epi=ops.EPI_SWIGLU_BF16)
            ops.gemm(a, L["wd"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
        return h

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        cfg = self.cfg
        h = self.forward_hidden(chunk, arena)
        if not getattr(chunk, "full_readout", False):
            return ops.final_norm_readout(h, chunk.final_rows, self.final_norm, cfg.rms_eps, self.answer_rows)
        R = chunk.final_rows.numel()
        normed = torch.empty(R, cfg.hidden, dtype=torch.bfloat16, device=h.device)
        ans = ops.final_norm_readout(h, chunk.final_rows, self.final_norm, cfg.rms_eps, self.answer_rows,
                                     normed=normed)
        return ops.head_readout(normed, self.head_bf16(), ans, getattr(chunk, "topk", False))
