"""Qwen3 decoder: the sm_100a kernel pipeline and its fp32 CPU statement.

Both take the same packed chunk (`quail_b200.engine.chunk.Chunk`) and the
same paged KV arena, and return the logits of the chunk's readout rows
against the retained answer rows of the LM head:

  embed -> [rmsnorm+quant -> QKV GEMM -> qk-norm+RoPE+KV write ->
            segmented paged attention (+quant) -> o GEMM (+residual) ->
            rmsnorm+quant -> gate_up GEMM (+SwiGLU+quant) -> down GEMM (+residual)] x L
        -> gather readout rows -> final norm -> answer-row logits

fp8 models fold those steps: the QKV epilogue does q/k norm, RoPE and the KV
write; the o / down GEMMs that update the residual also write it as MX e4m3
with per-row sums of squares, and the GEMM that reads it applies the row's
1 / rms (the RMSNorm weights are folded into the QKV and gate_up weights at
load), so no separate norm pass reads the residual stream.

The reference drives vLLM modules with its own loop
(quail/backends/quail/executor/models/qwen3.py:15-135, Engine primitives in
attention.py:432-1573); here every step is one of our kernels.
"""

from __future__ import annotations

import torch

from quail_b200.models.config import DecoderConfig
from quail_b200.models.weights import head_weight
from quail_b200.ops import reference as ref


class Qwen3Weights:
    """Per-layer fused device weights in the kernels' layouts.

    QKV rows are concatenated (q | k | v); gate/up rows are interleaved in
    64-row groups for the SwiGLU epilogue. fp8 models keep e4m3 weights with
    power-of-two 128x128 block scales as UE8M0 bytes in the MX atom layout
    (the tcgen05 block-scaled MMA's scale format); bf16 models keep bf16.
    """

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor], device, head_rows=None):
        from quail_b200.ops.quant import (dequantize_weight, interleave_gate_up, interleave_gate_up_mx,
                                          quantize_weight_mx)
        self.cfg = cfg
        self.device = device
        bf = torch.bfloat16
        self.embed = ckpt["model.embed_tokens.weight"].to(device=device, dtype=bf).contiguous()
        self.final_norm = ckpt["model.norm.weight"].to(device=device, dtype=bf)
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            L = {
                "ln1": ckpt[p + "input_layernorm.weight"].to(device=device, dtype=bf),
                "ln2": ckpt[p + "post_attention_layernorm.weight"].to(device=device, dtype=bf),
                "qn": ckpt[p + "self_attn.q_norm.weight"].to(device=device, dtype=bf),
                "kn": ckpt[p + "self_attn.k_norm.weight"].to(device=device, dtype=bf),
            }
            names = [p + "self_attn.q_proj", p + "self_attn.k_proj", p + "self_attn.v_proj"]
            if cfg.fp8:
                # fp8 checkpoints carry fp32 128x128 block scales; the tcgen05
                # block-scaled MMA takes power-of-two (UE8M0) scales, so each
                # projection is requantized once at load with the same blocks
                deq = lambda n: dequantize_weight(ckpt[n + ".weight"].to(device),  # noqa: E731
                                                  ckpt[n + ".weight_scale_inv"].to(device))
                # the RMSNorm weights fold into the K columns of the projections they feed:
                # (x / rms(x) * w) . W^T = (x . (W diag(w))^T) / rms(x), and the GEMMs apply 1 / rms
                ln1, ln2 = L["ln1"].float()[None, :], L["ln2"].float()[None, :]
                L["wqkv"], L["sqkv"] = quantize_weight_mx(torch.cat([deq(n) for n in names]) * ln1)
                L["wo"], L["so"] = quantize_weight_mx(deq(p + "self_attn.o_proj"))
                L["wgu"], L["sgu"] = interleave_gate_up_mx(torch.cat([deq(p + "mlp.gate_proj"),
                                                                      deq(p + "mlp.up_proj")]) * ln2)
                L["wd"], L["sd"] = quantize_weight_mx(deq(p + "mlp.down_proj"))
            else:
                L["wqkv"] = torch.cat([ckpt[n + ".weight"].to(bf) for n in names]).to(device).contiguous()
                L["wo"] = ckpt[p + "self_attn.o_proj.weight"].to(device=device, dtype=bf).contiguous()
                gu = torch.cat([ckpt[p + "mlp.gate_proj.weight"], ckpt[p + "mlp.up_proj.weight"]]).to(
                    device=device, dtype=bf)
                L["wgu"] = interleave_gate_up(gu)
                L["wd"] = ckpt[p + "mlp.down_proj.weight"].to(device=device, dtype=bf).contiguous()
            self.layers.append(L)
        self.head = head_weight(ckpt, cfg)
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.head_dim, cfg.rope_theta, device=device)
        if cfg.has_sae:
            self.sae_w = ckpt["sae.W_enc"].to(device=device, dtype=bf).contiguous()
            self.sae_b = ckpt["sae.b_enc"].to(device=device, dtype=torch.float32).contiguous()
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def head_bf16(self) -> torch.Tensor:
        """The whole LM head on the device in bf16 (for full-vocabulary readouts)."""
        if getattr(self, "_head_dev", None) is None:
            self._head_dev = self.head.to(device=self.device, dtype=torch.bfloat16).contiguous()
        return self._head_dev

    def set_answer_rows(self, token_ids) -> None:
        """Retain the LM-head rows of the answer tokens (yes/no or labels)."""
        ids = torch.as_tensor(list(token_ids), dtype=torch.long)
        rows = self.head.index_select(0, ids.to(self.head.device)).to(device=self.device, dtype=torch.bfloat16)
        old = getattr(self, "answer_rows", None)
        if old is not None and old.shape == rows.shape:
            old.copy_(rows)      # same buffer: captured decode graphs stay valid
        else:
            self.answer_rows = rows.contiguous()
        self.answer_ids = ids


class Qwen3Pipeline:
    """Forward pass of a packed chunk on the sm_100a kernels."""

    decision = None   # a decision model's head (models.decision.DecisionHead), set by the engine

    def __init__(self, cfg: DecoderConfig, weights: Qwen3Weights):
        assert cfg.head_dim == 128, "the kernels take head_dim 128"
        self.cfg = cfg
        self.w = weights
        self.scale = ref.softmax_scale(cfg.head_dim)
        # the tcgen05 attention packs four q heads of one KV head per CTA
        self.tc_attention = (cfg.num_q_heads // cfg.num_kv_heads) % 4 == 0

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        cfg, w = self.cfg, self.w
        T = chunk.num_tokens
        dev = w.device
        h = ops.embed_gather(chunk.ids, w.embed)  # residual stream, bf16 [T, H]
        fp8 = cfg.fp8
        H = cfg.hidden
        if fp8:
            # the residual stream's RMSNorms run inside the GEMMs: the GEMM that writes h also
            # writes it as MX e4m3 with per-128-column sums of squares, and the next GEMM
            # scales its rows by 1 / rms (the norm weights are folded into its weights)
            x8, xs, ss = ops.quant_mx_ss(h)
        n_layers = len(w.layers)
        for li, L in enumerate(w.layers):
            kc, vc = arena.layer(li)
            if fp8:
                # K1 + K4: QKV GEMM whose epilogue norms, rotates and writes K/V to the arena
                q = ops.gemm_mx_qkv_rope(x8, xs, L["wqkv"], L["sqkv"], chunk.positions, chunk.slots, L["qn"],
                                         L["kn"], w.cos_sin, kc, vc, cfg.num_q_heads, cfg.num_kv_heads, cfg.rms_eps,
                                         row_ss=ops.row_rinv(ss, H, cfg.rms_eps))
                o8, os_ = ops.chunk_attention(q, kc, vc, chunk, self.scale, mx=True, tc=self.tc_attention)
                x8 = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=dev)
                xs = torch.empty(ops.sf_bytes(T, H), dtype=torch.uint8, device=dev)
                ss = torch.empty(T, H // 128, dtype=torch.float32, device=dev)
                ops.gemm_mx(o8, os_, L["wo"], L["so"], epi=ops.EPI_RESIDUAL_MX, out=h, residual=h, xq=x8, xq_sf=xs,
                            ss_out=ss)
                # one 1 / rms per row for the whole gate_up GEMM (its epilogue then reads one float)
                a8, as_ = ops.gemm_mx(x8, xs, L["wgu"], L["sgu"], epi=ops.EPI_SWIGLU_FP8,
                                      row_ss=ops.row_rinv(ss, H, cfg.rms_eps), eps=cfg.rms_eps)
                if li == n_layers - 1:
                    ops.gemm_mx(a8, as_, L["wd"], L["sd"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
                    continue
                x8 = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=dev)
                xs = torch.empty(ops.sf_bytes(T, H), dtype=torch.uint8, device=dev)
                ss = torch.empty(T, H // 128, dtype=torch.float32, device=dev)
                ops.gemm_mx(a8, as_, L["wd"], L["sd"], epi=ops.EPI_RESIDUAL_MX, out=h, residual=h, xq=x8, xq_sf=xs,
                            ss_out=ss)
                continue
            x = ops.rmsnorm_quant(h, L["ln1"], cfg.rms_eps, fp8=False)
            qkv = ops.gemm(x, L["wqkv"])
            q = ops.qk_norm_rope_kv(qkv, chunk.positions, L["qn"], L["kn"], w.cos_sin, chunk.slots, kc, vc,
                                    cfg.num_q_heads, cfg.num_kv_heads, cfg.rms_eps)
            o = ops.chunk_attention(q, kc, vc, chunk, self.scale, mx=False, tc=self.tc_attention)
            ops.gemm(o, L["wo"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
            x = ops.rmsnorm_quant(h, L["ln2"], cfg.rms_eps, fp8=False)
            a = ops.gemm(x, L["wgu"], epi=ops.EPI_SWIGLU_BF16)
            ops.gemm(a, L["wd"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
        del T, dev, H
        if cfg.has_sae:
            # resid_post of the last loaded layer -> packed SAE features per readout row
            return ops.sae_features(h.index_select(0, chunk.final_rows.long()), w.sae_w, w.sae_b, cfg.sae_keep)
        if self.decision is not None:
            # decision model: the head's projections of the final-normed rows
            normed = torch.empty(chunk.final_rows.numel(), cfg.hidden, dtype=torch.bfloat16, device=h.device)
            ops.final_norm_readout(h, chunk.final_rows, w.final_norm, cfg.rms_eps, w.answer_rows, normed=normed)
            return self.decision.features(normed)
        if not getattr(chunk, "full_readout", False):
            return ops.final_norm_readout(h, chunk.final_rows, w.final_norm, cfg.rms_eps, w.answer_rows)
        R = chunk.final_rows.numel()
        normed = torch.empty(R, cfg.hidden, dtype=torch.bfloat16, device=h.device)
        ans = ops.final_norm_readout(h, chunk.final_rows, w.final_norm, cfg.rms_eps, w.answer_rows, normed=normed)
        return ops.head_readout(normed, w.head_bf16(), ans, getattr(chunk, "topk", False))


class Qwen3Reference:
    """fp32 PyTorch forward over the same chunk and arena (CPU or GPU).

    Weights are dequantized from the checkpoint, so an fp8 checkpoint gives
    the math the kernels approximate (activations stay fp32 here).
    """

    decision = None

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor], device="cpu", head_rows=None,
                 dtype=torch.float32, emulate_kernels: bool = False):
        self.cfg = cfg
        self.device = device
        self.dtype = dtype
        # round where the kernels round: bf16 residual stream, q/k/v and KV;
        # e4m3 + 1x128 scales on every GEMM input of an fp8 model
        self.emulate = emulate_kernels
        f = lambda t: t.to(device=device, dtype=dtype)  # noqa: E731
        if self.emulate and cfg.fp8:
            from quail_b200.ops.quant import dequantize_mx, quantize_weight_mx

            def dequantized(ck, name):  # noqa: F811 - the kernels' power-of-two requantization
                from quail_b200.models.weights import dequantized as plain
                return dequantize_mx(*quantize_weight_mx(plain(ck, name).to(device)))
        else:
            from quail_b200.models.weights import dequantized
        self.embed = f(ckpt["model.embed_tokens.weight"])
        self.final_norm = f(ckpt["model.norm.weight"])
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            L = {
                "ln1": f(ckpt[p + "input_layernorm.weight"]), "ln2": f(ckpt[p + "post_attention_layernorm.weight"]),
                "qn": f(ckpt[p + "self_attn.q_norm.weight"]), "kn": f(ckpt[p + "self_attn.k_norm.weight"]),
                "wq": f(dequantized(ckpt, p + "self_attn.q_proj")), "wk": f(dequantized(ckpt, p + "self_attn.k_proj")),
                "wv": f(dequantized(ckpt, p + "self_attn.v_proj")), "wo": f(dequantized(ckpt, p + "self_attn.o_proj")),
            }
            if cfg.is_moe:
                # router (kept bf16 in checkpoints) and the experts' SwiGLU weights
                L["router"] = f(ckpt[p + "mlp.gate.weight"])
                L["experts"] = [tuple(f(dequantized(ckpt, p + f"mlp.experts.{e}.{n}"))
                                      for n in ("gate_proj", "up_proj", "down_proj"))
                                for e in range(cfg.num_experts)]
            else:
                L.update(wg=f(dequantized(ckpt, p + "mlp.gate_proj")), wu=f(dequantized(ckpt, p + "mlp.up_proj")),
                         wd=f(dequantized(ckpt, p + "mlp.down_proj")))
            self.layers.append(L)
        self.head = f(head_weight(ckpt, cfg))
        if cfg.has_sae:
            self.sae_w = f(ckpt["sae.W_enc"])
            self.sae_b = f(ckpt["sae.b_enc"])
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.head_dim, cfg.rope_theta, device=device)
        self.scale = ref.softmax_scale(cfg.head_dim)
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def set_answer_rows(self, token_ids) -> None:
        ids = torch.as_tensor(list(token_ids), dtype=torch.long, device=self.head.device)
        self.answer_rows = self.head.index_select(0, ids)
        self.answer_ids = ids.cpu()

    def _q(self, x: torch.Tensor) -> torch.Tensor:
        """fake-quantize a GEMM input the way the fp8 kernels do."""
        if not (self.emulate and self.cfg.fp8):
            return x
        from quail_b200.ops.quant import dequantize_mx, quantize_act_mx
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        return dequantize_mx(*quantize_act_mx(x2)).reshape(shape)

    def _bf(self, x: torch.Tensor) -> torch.Tensor:
        return x.bfloat16().float() if self.emulate else x

    @torch.no_grad()
    def hidden_chunk(self, chunk, arena) -> torch.Tensor:
        cfg = self.cfg
        T = chunk.num_tokens
        h = self._bf(self.embed[chunk.ids.long()])
        QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        for li, L in enumerate(self.layers):
            kc, vc = arena.layer(li)
            x = self._q(self._bf(ref.rmsnorm(h, L["ln1"], cfg.rms_eps)))
            q = self._bf(x @ L["wq"].t()).view(T, QH, D)
            k = self._bf(x @ L["wk"].t()).view(T, KH, D)
            v = self._bf(x @ L["wv"].t()).view(T, KH, D)
            q = self._bf(ref.rope_neox(ref.rmsnorm(q, L["qn"], cfg.rms_eps), chunk.positions, self.cos_sin))
            k = ref.rope_neox(ref.rmsnorm(k, L["kn"], cfg.rms_eps), chunk.positions, self.cos_sin)
            ok = chunk.slots >= 0
            slots = chunk.slots[ok].long()
            kc.view(-1, KH, D)[slots] = self._bf(k[ok]).to(kc.dtype)
            vc.view(-1, KH, D)[slots] = self._bf(v[ok]).to(vc.dtype)
            tree = getattr(chunk, "tree", None)
            if tree is not None:
                # the tree path: two reads merged by their log-sum-exps (the same sum, reordered)
                o = ref.tree_attention(q, kc, vc, chunk.seqs, chunk.page_list, tree, self.scale).to(h.dtype)
            else:
                o = ref.segmented_attention(q, kc, vc, chunk.seqs, chunk.page_list, self.scale).to(h.dtype)
            o = self._q(o) if self.cfg.fp8 else self._bf(o)
            h = self._bf(h + o @ L["wo"].t())
            x = self._q(self._bf(ref.rmsnorm(h, L["ln2"], cfg.rms_eps)))
            if cfg.is_moe:
                h = self._bf(h + self._moe(x, self._bf(ref.rmsnorm(h, L["ln2"], cfg.rms_eps)), L))
                continue
            a = ref.silu_mul(x @ L["wg"].t(), x @ L["wu"].t())
            a = self._q(a) if self.cfg.fp8 else self._bf(a)
            h = self._bf(h + a @ L["wd"].t())
        return h

    def _moe(self, x: torch.Tensor, xr: torch.Tensor, L) -> torch.Tensor:
        """Softmax router, top-k with renormalized weights, SwiGLU experts (Qwen3-MoE)."""
        logits = self._bf(xr @ L["router"].t())
        ids, wts = ref.moe_route(logits, self.cfg.top_k)
        out = torch.zeros_like(x)
        for e, (wg, wu, wd) in enumerate(L["experts"]):
            rows, ks = (ids == e).nonzero(as_tuple=True)
            if rows.numel() == 0:
                continue
            xe = x[rows]
            a = ref.silu_mul(xe @ wg.t(), xe @ wu.t())
            a = self._q(a) if self.cfg.fp8 else self._bf(a)
            # each weighted expert row is stored in bf16 before the sum over k
            out.index_add_(0, rows, self._bf((a @ wd.t()) * wts[rows, ks][:, None]))
        return out

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        h = self.hidden_chunk(chunk, arena)
        rows = h[chunk.final_rows.long()]
        if self.cfg.has_sae:
            x = self._bf(rows) if self.emulate else rows
            return ref.sae_features(x, self.sae_w, self.sae_b, self.cfg.sae_keep)
        normed = ref.rmsnorm(rows, self.final_norm, self.cfg.rms_eps)
        if self.decision is not None:
            return self.decision.features(normed)
        ans = (normed @ self.answer_rows.t()).float()
        if not getattr(chunk, "full_readout", False):
            return ans
        full = (normed @ self.head.t()).float()
        return ref.head_readout(full, ans, getattr(chunk, "topk", False))
