"""Qwen3.5 hybrid decoder on the sm_100a kernels (bf16 weights).

Per layer, on our kernels (fp8 checkpoints: attention and MLP GEMMs on the
block-scaled fp8 tcgen05 GEMM with MX activations, Gated DeltaNet in bf16):
  RMSNorm (bf16 out) ->
    Gated DeltaNet: in-projection GEMM [qkv | z | b | a] -> gdn_layer (causal
      conv + L2 norm, delta-rule recurrence over the state slots, gated RMSNorm)
      -> out_proj GEMM (+ residual)
    gated attention: q|gate|k|v GEMM -> q/k norm + partial RoPE + KV write ->
      small-tile paged attention with the sigmoid gate -> o_proj GEMM (+ residual)
  -> RMSNorm -> gate_up GEMM (+ SwiGLU) -> down GEMM (+ residual)
then the final norm and the readout. The zero-centered norms (scale 1 + w)
are folded into the weights at load.

Reference: quail/backends/quail/executor/models/qwen3_5.py:36-391 (the
reference's Qwen3.5 pipeline over vLLM modules).
"""

from __future__ import annotations

import os

import torch

from quail_b200.models.config import DecoderConfig
from quail_b200.models.weights import dequantized, head_weight
from quail_b200.ops import reference as ref


def _pad_rows(w: torch.Tensor, multiple: int = 16) -> torch.Tensor:
    n = w.shape[0]
    m = -(-n // multiple) * multiple
    if m == n:
        return w.contiguous()
    out = torch.zeros(m, w.shape[1], dtype=w.dtype, device=w.device)
    out[:n] = w
    return out


class Qwen35Pipeline:
    """Forward pass of a packed chunk of a Qwen3.5 hybrid on the GPU kernels."""

    images = None           # engine.images.ImageStore of a model with a vision tower

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor], device, head_rows=None,
                 max_tokens: int = 16384):
        from quail_b200.ops.quant import (interleave_gate_up, interleave_gate_up_mx, quantize_nvfp4,
                                          quantize_weight_mx)
        assert cfg.is_hybrid
        self.cfg = cfg
        self.device = device
        bf = torch.bfloat16
        dev = device
        off = 1.0 if cfg.norm_offset else 0.0

        def norm_w(t):
            return (t.float() + off).to(device=dev, dtype=bf)

        def fp32(name):
            return dequantized(ckpt, name).to(device=dev)

        def proj(name):
            return fp32(name).to(bf)

        # fp8 checkpoints: attention and MLP projections on the block-scaled fp8
        # GEMM (requantized to power-of-two 128x128 blocks); the Gated DeltaNet
        # projections stay bf16
        self.fp8 = cfg.fp8

        self.embed = ckpt["model.embed_tokens.weight"].to(device=dev, dtype=bf).contiguous()
        self.final_norm = norm_w(ckpt["model.norm.weight"])
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            L = {"ln1": norm_w(ckpt[p + "input_layernorm.weight"]),
                 "ln2": norm_w(ckpt[p + "post_attention_layernorm.weight"])}
            if cfg.kind(i) == "gdn":
                q = p + "linear_attn."
                L["win"] = _pad_rows(torch.cat([proj(q + "in_proj_qkv"), proj(q + "in_proj_z"),
                                                proj(q + "in_proj_b"), proj(q + "in_proj_a")]))
                L["wout"] = proj(q + "out_proj").contiguous()
                L["conv"] = ckpt[q + "conv1d.weight"][:, 0, :].to(device=dev, dtype=torch.float32).contiguous()
                L["A_log"] = ckpt[q + "A_log"].to(device=dev, dtype=torch.float32).contiguous()
                L["dt_bias"] = ckpt[q + "dt_bias"].to(device=dev, dtype=torch.float32).contiguous()
                L["norm"] = ckpt[q + "norm.weight"].to(device=dev, dtype=bf).contiguous()
            else:
                q = p + "self_attn."
                qkv = torch.cat([fp32(q + "q_proj"), fp32(q + "k_proj"), fp32(q + "v_proj")])
                if self.fp8:
                    L["wqkv"], L["sqkv"] = quantize_weight_mx(qkv)
                    L["wo"], L["so"] = quantize_weight_mx(fp32(q + "o_proj"))
                else:
                    L["wqkv"] = _pad_rows(qkv.to(bf))
                    L["wo"] = proj(q + "o_proj").contiguous()
                L["qn"] = ckpt[q + "q_norm.weight"].to(device=dev, dtype=bf).contiguous()
                L["kn"] = ckpt[q + "k_norm.weight"].to(device=dev, dtype=bf).contiguous()
            if cfg.is_moe:
                self._moe_weights(L, p + "mlp.", fp32, quantize_weight_mx, interleave_gate_up_mx)
                self.layers.append(L)
                continue
            gu = torch.cat([fp32(p + "mlp.gate_proj"), fp32(p + "mlp.up_proj")])
            if cfg.mlp_fp4:
                # NVFP4 MLP: gate | up rows (not interleaved: the SwiGLU runs in the
                # activation quantizer), one global scale per weight
                L["wgu4"] = quantize_nvfp4(gu)
                L["wd4"] = quantize_nvfp4(fp32(p + "mlp.down_proj"))
                self.layers.append(L)
                continue
            if self.fp8:
                L["wgu"], L["sgu"] = interleave_gate_up_mx(gu)
                L["wd"], L["sd"] = quantize_weight_mx(fp32(p + "mlp.down_proj"))
            else:
                L["wgu"] = interleave_gate_up(gu.to(bf))
                L["wd"] = proj(p + "mlp.down_proj").contiguous()
            self.layers.append(L)
        self.head = head_weight(ckpt, cfg)
        if cfg.has_sae:
            self.sae_w = ckpt["sae.W_enc"].to(device=dev, dtype=bf).contiguous()
            self.sae_b = ckpt["sae.b_enc"].to(device=dev, dtype=torch.float32).contiguous()
        # Gated DeltaNet recurrence: 0 = chunked tensor-core form for prefill passes, 1 = per token
        self.gdn_mode = int(os.environ.get("QB_GDN_MODE", "0"))
        self.ep = None
        if cfg.is_moe:
            from quail_b200.parallel.ep import EPState
            self.ep = EPState(cfg, max_tokens, dev, None)
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.rotary_dim, cfg.rope_theta, device=dev)
        self.scale = ref.softmax_scale(cfg.head_dim)
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def _moe_weights(self, L, m, fp32, quantize_weight_mx, interleave_gate_up_mx):
        """Router (bf16), the routed experts stacked in the MX layout the grouped GEMMs read, and
        the shared expert (MX) with its gate row (bf16, padded to 16 rows for the GEMM)."""
        cfg, dev = self.cfg, self.device
        L["router"] = fp32(m + "gate").to(torch.bfloat16).contiguous()
        gq, gs, dq, ds = [], [], [], []
        for e in range(cfg.num_experts):
            q, sc = interleave_gate_up_mx(torch.cat([fp32(m + f"experts.{e}.gate_proj"),
                                                     fp32(m + f"experts.{e}.up_proj")]))
            gq.append(q)
            gs.append(sc)
            q, sc = quantize_weight_mx(fp32(m + f"experts.{e}.down_proj"))
            dq.append(q)
            ds.append(sc)
        L["wgu"], L["sgu"] = torch.cat(gq).contiguous(), torch.cat(gs).contiguous()
        L["wd"], L["sd"] = torch.cat(dq).contiguous(), torch.cat(ds).contiguous()
        if cfg.shared_intermediate:
            L["wgu_s"], L["sgu_s"] = interleave_gate_up_mx(torch.cat([fp32(m + "shared_expert.gate_proj"),
                                                                      fp32(m + "shared_expert.up_proj")]))
            L["wd_s"], L["sd_s"] = quantize_weight_mx(fp32(m + "shared_expert.down_proj"))
            g = torch.zeros(16, cfg.hidden, dtype=torch.bfloat16, device=dev)
            g[0] = fp32(m + "shared_expert_gate")[0].to(torch.bfloat16)
            L["wsg"] = g

    def _moe_mlp(self, h, L):
        """h += sigmoid(x . w_gate) * shared(x) + sum_k w_k expert_k(x), x = norm(h)."""
        from quail_b200 import ops
        cfg = self.cfg
        x8, xs = ops.rmsnorm_quant_mx(h, L["ln2"], cfg.rms_eps)
        xb = ops.rmsnorm_quant(h, L["ln2"], cfg.rms_eps, fp8=False)
        if "wgu_s" in L:
            a8, as_ = ops.gemm_mx(x8, xs, L["wgu_s"], L["sgu_s"], epi=ops.EPI_SWIGLU_FP8)
            sh = ops.gemm_mx(a8, as_, L["wd_s"], L["sd_s"])
            g = ops.gemm(xb, L["wsg"])
            h.add_(sh * torch.sigmoid(g[:, :1].float()).to(sh.dtype))
        self.ep.forward(x8, xs, xb, h, L, next_norm=None, eps=cfg.rms_eps)

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
        dev = self.device
        QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        Hk, Hv, dk, dv = cfg.gdn_key_heads, cfg.gdn_value_heads, cfg.gdn_key_dim, cfg.gdn_value_dim
        if self.cfg.has_vision and self.images is not None and getattr(chunk, "rope3", None) is not None:
            from quail_b200.models.qwen3_5 import image_embeddings
            h = image_embeddings(chunk.ids, self.embed, self.images).contiguous()
        else:
            h = ops.embed_gather(chunk.ids, self.embed)
        gi = ai = 0
        for i, L in enumerate(self.layers):
            if cfg.kind(i) == "gdn":
                x = ops.rmsnorm_quant(h, L["ln1"], cfg.rms_eps, fp8=False)
                p = ops.gemm(x, L["win"])
                conv_out = torch.empty(T, cfg.gdn_conv_dim, dtype=torch.float32, device=dev)
                o = torch.empty(T, Hv * dv, dtype=torch.float32, device=dev)
                y = torch.empty(T, Hv * dv, dtype=torch.bfloat16, device=dev)
                ops.count_launch(3)
                C.gdn_layer(p, L["conv"], L["A_log"], L["dt_bias"], L["norm"], chunk.seqs, chunk.state_io,
                            arena.states["conv"], arena.states["ssm"], gi, Hk, Hv, dk, dv, cfg.rms_eps, conv_out, o, y,
                            self.gdn_mode)
                ops.gemm(y, L["wout"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
                gi += 1
            else:
                if self.fp8:
                    x8, xs = ops.rmsnorm_quant_mx(h, L["ln1"], cfg.rms_eps)
                    p = ops.gemm_mx(x8, xs, L["wqkv"], L["sqkv"])
                else:
                    p = ops.gemm(ops.rmsnorm_quant(h, L["ln1"], cfg.rms_eps, fp8=False), L["wqkv"])
                kc, vc = arena.layer(ai)
                q = torch.empty(T, QH, D, dtype=torch.bfloat16, device=dev)
                ops.count_launch(1)
                rope3 = getattr(chunk, "rope3", None)
                sec = cfg.mrope_sections if rope3 is not None else (0, 0, 0)
                C.hybrid_qk_rope_kv(p, QH, KH, cfg.attn_output_gate, rope3 if rope3 is not None else chunk.positions,
                                    L["qn"], L["kn"], cfg.norm_offset, self.cos_sin, chunk.slots, kc, vc, q,
                                    cfg.rms_eps, sec[1], sec[2])
                o = torch.empty(T, QH * D, dtype=torch.bfloat16, device=dev)
                gate = p[:, D:] if cfg.attn_output_gate else None
                ops.small_attention(q, kc, vc, chunk.seqs, chunk.tiles, chunk.dseqs, chunk.page_list, self.scale, o,
                                  gate, 2 * D)
                if self.fp8:
                    o8, os_ = ops.quant_rows_mx(o)
                    ops.gemm_mx(o8, os_, L["wo"], L["so"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
                else:
                    ops.gemm(o, L["wo"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
                ai += 1
            if self.ep is not None:
                self._moe_mlp(h, L)
                continue
            if "wgu4" in L:
                x = ops.rmsnorm_quant(h, L["ln2"], cfg.rms_eps, fp8=False)
                q, sf, rs = ops.quant_rows_nvfp4(x)
                wq, ws, wg = L["wgu4"]
                gu = ops.gemm_nvfp4(q, sf, wq, ws, wg, row_scale=rs)
                q, sf, rs = ops.quant_rows_nvfp4(gu, swiglu=True)
                wq, ws, wg = L["wd4"]
                ops.gemm_nvfp4(q, sf, wq, ws, wg, row_scale=rs, epi=ops.EPI_RESIDUAL, out=h, residual=h)
                continue
            if self.fp8:
                x8, xs = ops.rmsnorm_quant_mx(h, L["ln2"], cfg.rms_eps)
                a8, as_ = ops.gemm_mx(x8, xs, L["wgu"], L["sgu"], epi=ops.EPI_SWIGLU_FP8)
                ops.gemm_mx(a8, as_, L["wd"], L["sd"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
                continue
            x = ops.rmsnorm_quant(h, L["ln2"], cfg.rms_eps, fp8=False)
            a = ops.gemm(x, L["wgu"], epi=ops.EPI_SWIGLU_BF16)
            ops.gemm(a, L["wd"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
        return h

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        cfg = self.cfg
        h = self.forward_hidden(chunk, arena)
        if cfg.has_sae:
            return ops.sae_features(h.index_select(0, chunk.final_rows.long()), self.sae_w, self.sae_b, cfg.sae_keep)
        if not getattr(chunk, "full_readout", False):
            return ops.final_norm_readout(h, chunk.final_rows, self.final_norm, cfg.rms_eps, self.answer_rows)
        R = chunk.final_rows.numel()
        normed = torch.empty(R, cfg.hidden, dtype=torch.bfloat16, device=h.device)
        ans = ops.final_norm_readout(h, chunk.final_rows, self.final_norm, cfg.rms_eps, self.answer_rows,
                                     normed=normed)
        return ops.head_readout(normed, self.head_bf16(), ans, getattr(chunk, "topk", False))
