"""Qwen3.5 hybrid decoder: Gated DeltaNet layers and gated full attention.

Layer kinds follow `DecoderConfig.layer_kinds` (three Gated DeltaNet layers per
full-attention layer in the released models). Every layer is
`h += mixer(norm(h)); h += SwiGLU(norm(h))` with zero-centered RMSNorms
(scale 1 + w).

Gated DeltaNet (per token t, value head h; q/k heads shared by
gdn_value_heads / gdn_key_heads value heads):

  x_qkv = causal depthwise conv (width w) over in_proj_qkv(x), then SiLU
  q, k  = L2-normalized per head (q also scaled by d_k^-1/2); v as is
  g     = -exp(A_log) * softplus(in_proj_a(x) + dt_bias)     (log decay)
  beta  = sigmoid(in_proj_b(x))
  S     = exp(g) * S;  S += beta * k (v - S^T k)^T;  o = S^T q     (S: d_k x d_v)
  out   = out_proj(RMSNorm(o) * norm_w * silu(in_proj_z(x)))

The state of a sequence (conv window of its last w-1 inputs and S per head)
lives in the arena's state slot of its key; a sequence starts from its own
slot when it continues its key, else from the slot of the last segment it
reads (the shared prefix for a document, the document for a question).

Gated attention: q_proj emits [q | gate] per head; q/k RMSNorm (1 + w) per
head, RoPE on the first `rotary_dim` dims (NeoX halves), paged attention,
output * sigmoid(gate), o_proj.

Reference: the reference runs Qwen3.5 through vLLM with its own GDN phases
and checkpoint slots (quail/backends/quail/executor/models/qwen3_5.py:36-391,
gdn.py:27-1088); this module states the same math in fp32 PyTorch.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from quail_b200.models.config import DecoderConfig
from quail_b200.models.weights import head_weight
from quail_b200.ops import reference as ref


def rmsnorm_offset(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm with zero-centered weights: x / rms(x) * (1 + w)."""
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())


def rope_partial(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, rotary_dim: int,
                 sections=None) -> torch.Tensor:
    """NeoX RoPE on the first `rotary_dim` dims of each head; the rest pass through. [T, 3]
    positions (with `sections`) rotate by interleaved multimodal RoPE (ops.reference.rope_neox_3d)."""
    def rot(y):
        if positions.dim() == 2:
            return ref.rope_neox_3d(y, positions, cos_sin, sections)
        return ref.rope_neox(y, positions, cos_sin)
    if rotary_dim == x.shape[-1]:
        return rot(x)
    return torch.cat([rot(x[..., :rotary_dim]), x[..., rotary_dim:]], dim=-1)


def image_embeddings(ids: torch.Tensor, embed: torch.Tensor, images) -> torch.Tensor:
    """Token embeddings; ids at or above the image token base take their rows of the region's
    vision-tower output (`images`: engine.images.ImageStore) instead of the text table."""
    from quail_b200.engine.images import IMAGE_TOKEN_BASE
    ids = ids.long()
    img = ids >= IMAGE_TOKEN_BASE
    h = embed[torch.where(img, torch.zeros_like(ids), ids)]
    if images is not None and bool(img.any()):
        table = images.table(h.device, h.dtype)
        h[img] = table[ids[img] - IMAGE_TOKEN_BASE]
    return h


def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """(g, beta) per token and value head: g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)."""
    g = -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())
    return g, torch.sigmoid(b.float())


def causal_conv(x: torch.Tensor, window: torch.Tensor, w: torch.Tensor):
    """Depthwise causal conv of x [n, C] continuing `window` [w-1, C]; weights w [C, width].

    Returns (SiLU(conv) [n, C], the new window: the last w-1 inputs)."""
    width = w.shape[1]
    full = torch.cat([window.to(x.dtype), x], dim=0)                 # [w-1+n, C]
    n = x.shape[0]
    out = torch.zeros_like(x)
    for j in range(width):
        out += full[j:j + n] * w[:, j]
    return F.silu(out), full[-(width - 1):].clone()


def delta_rule(q, k, v, g, beta, S):
    """Gated delta rule over n tokens. q, k [n, Hv, dk] (normalized, q scaled), v [n, Hv, dv],
    g, beta [n, Hv], S [Hv, dk, dv] (updated in place). Returns o [n, Hv, dv]."""
    n = q.shape[0]
    out = torch.empty(n, v.shape[1], v.shape[2], dtype=S.dtype, device=S.device)
    for t in range(n):
        S.mul_(torch.exp(g[t])[:, None, None])
        kv = torch.einsum("hk,hkv->hv", k[t], S)
        delta = (v[t] - kv) * beta[t][:, None]
        S.add_(k[t][:, :, None] * delta[:, None, :])
        out[t] = torch.einsum("hk,hkv->hv", q[t], S)
    return out


class Qwen35Reference:
    """fp32 PyTorch forward of a Qwen3.5 hybrid over packed chunks (CPU or GPU).

    Same contract as `Qwen3Reference`: forward_chunk(chunk, arena) returns the
    readout rows' logits against the retained answer rows (plus argmax and
    log-sum-exp columns for full readouts). The arena holds KV pages for the
    attention layers (layer index -> position in cfg.attn_layers) and state
    slots for the Gated DeltaNet layers.
    """

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor], device="cpu", head_rows=None,
                 dtype=torch.float32, emulate_kernels: bool = False):
        from quail_b200.models.weights import dequantized as plain
        assert cfg.is_hybrid
        self.cfg = cfg
        self.device = device
        # emulate_kernels (fp8 checkpoints): the kernels' power-of-two weight
        # requantization, e4m3 + 1x32 scales on every fp8 GEMM input, and a
        # bf16 residual stream; the Gated DeltaNet projections stay as stored
        self.emulate = emulate_kernels and cfg.fp8
        self.fp4 = self.emulate and cfg.mlp_fp4

        def dequantized(ck, name):
            if not self.emulate or ".linear_attn." in name or ck.get(name + ".weight_scale_inv") is None:
                return plain(ck, name)
            from quail_b200.ops.quant import dequantize_mx, quantize_weight_mx
            return dequantize_mx(*quantize_weight_mx(plain(ck, name).to(device)))
        f = lambda t: t.to(device=device, dtype=dtype)  # noqa: E731
        self.embed = f(ckpt["model.embed_tokens.weight"])
        self.final_norm = f(ckpt["model.norm.weight"])
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            L = {"ln1": f(ckpt[p + "input_layernorm.weight"]), "ln2": f(ckpt[p + "post_attention_layernorm.weight"])}
            if cfg.is_moe:
                m = p + "mlp."
                L["router"] = f(ckpt[m + "gate.weight"])
                L["experts"] = [(f(dequantized(ckpt, m + f"experts.{e}.gate_proj")),
                                 f(dequantized(ckpt, m + f"experts.{e}.up_proj")),
                                 f(dequantized(ckpt, m + f"experts.{e}.down_proj"))) for e in range(cfg.num_experts)]
                if cfg.shared_intermediate:
                    L["shared"] = (f(dequantized(ckpt, m + "shared_expert.gate_proj")),
                                   f(dequantized(ckpt, m + "shared_expert.up_proj")),
                                   f(dequantized(ckpt, m + "shared_expert.down_proj")))
                    L["shared_gate"] = f(ckpt[m + "shared_expert_gate.weight"])
            elif self.fp4:
                # the kernels' NVFP4 weights: gate | up quantized together, down alone
                from quail_b200.models.weights import dequantized as plain
                from quail_b200.ops.quant import dequantize_nvfp4, quantize_nvfp4
                gu = torch.cat([plain(ckpt, p + "mlp.gate_proj"), plain(ckpt, p + "mlp.up_proj")]).to(device)
                gu = dequantize_nvfp4(*quantize_nvfp4(gu), gu.shape[1])
                wd = plain(ckpt, p + "mlp.down_proj").to(device)
                L.update(wg=f(gu[:gu.shape[0] // 2]), wu=f(gu[gu.shape[0] // 2:]),
                         wd=f(dequantize_nvfp4(*quantize_nvfp4(wd), wd.shape[1])))
            else:
                L.update(wg=f(dequantized(ckpt, p + "mlp.gate_proj")), wu=f(dequantized(ckpt, p + "mlp.up_proj")),
                         wd=f(dequantized(ckpt, p + "mlp.down_proj")))
            if cfg.kind(i) == "gdn":
                q = p + "linear_attn."
                L.update(qkv=f(dequantized(ckpt, q + "in_proj_qkv")), z=f(dequantized(ckpt, q + "in_proj_z")),
                         b=f(dequantized(ckpt, q + "in_proj_b")), a=f(dequantized(ckpt, q + "in_proj_a")),
                         out=f(dequantized(ckpt, q + "out_proj")), conv=f(ckpt[q + "conv1d.weight"][:, 0, :]),
                         A_log=f(ckpt[q + "A_log"]), dt_bias=f(ckpt[q + "dt_bias"]),
                         norm=f(ckpt[q + "norm.weight"]))
            else:
                q = p + "self_attn."
                L.update(wq=f(dequantized(ckpt, q + "q_proj")), wk=f(dequantized(ckpt, q + "k_proj")),
                         wv=f(dequantized(ckpt, q + "v_proj")), wo=f(dequantized(ckpt, q + "o_proj")),
                         qn=f(ckpt[q + "q_norm.weight"]), kn=f(ckpt[q + "k_norm.weight"]))
            self.layers.append(L)
        self.head = f(head_weight(ckpt, cfg))
        if cfg.has_sae:
            self.sae_w, self.sae_b = f(ckpt["sae.W_enc"]), f(ckpt["sae.b_enc"])
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.rotary_dim, cfg.rope_theta, device=device)
        self.scale = ref.softmax_scale(cfg.head_dim)
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def set_answer_rows(self, token_ids) -> None:
        ids = torch.as_tensor(list(token_ids), dtype=torch.long, device=self.head.device)
        self.answer_rows = self.head.index_select(0, ids)
        self.answer_ids = ids.cpu()

    # ------------------------------------------------------------ mixers
    def _gdn(self, x, L, gi, chunk, arena):
        """Gated DeltaNet layer gi (index among the GDN layers) over every sequence of the chunk."""
        cfg = self.cfg
        Hk, Hv, dk, dv = cfg.gdn_key_heads, cfg.gdn_value_heads, cfg.gdn_key_dim, cfg.gdn_value_dim
        conv_s, ssm_s = arena.states["conv"], arena.states["ssm"]
        mixed = x @ L["qkv"].t()
        z = x @ L["z"].t()
        g, beta = gdn_gates(x @ L["a"].t(), x @ L["b"].t(), L["A_log"], L["dt_bias"])
        out = torch.empty(x.shape[0], Hv * dv, dtype=x.dtype, device=x.device)
        seqs = chunk.seqs.cpu() if chunk.seqs.is_cuda else chunk.seqs
        sio = chunk.state_io.cpu() if chunk.state_io.is_cuda else chunk.state_io
        for s in range(seqs.shape[0]):
            q0, n = int(seqs[s, 0]), int(seqs[s, 1])
            src, dst = int(sio[s, 0]), int(sio[s, 1])
            if src >= 0:
                window, S = conv_s[src, gi].clone(), ssm_s[src, gi].clone()
            else:
                window = torch.zeros_like(conv_s[0, gi])
                S = torch.zeros_like(ssm_s[0, gi])
            c, window = causal_conv(mixed[q0:q0 + n], window, L["conv"])
            qq = c[:, :Hk * dk].view(n, Hk, dk)
            kk = c[:, Hk * dk:2 * Hk * dk].view(n, Hk, dk)
            vv = c[:, 2 * Hk * dk:].view(n, Hv, dv)
            qq = F.normalize(qq.float(), dim=-1) * dk ** -0.5
            kk = F.normalize(kk.float(), dim=-1)
            rep = Hv // Hk
            qq, kk = qq.repeat_interleave(rep, 1), kk.repeat_interleave(rep, 1)
            o = delta_rule(qq, kk, vv.float(), g[q0:q0 + n], beta[q0:q0 + n], S)
            conv_s[dst, gi] = window.float()
            ssm_s[dst, gi] = S
            o = ref.rmsnorm(o, L["norm"], cfg.rms_eps) * F.silu(z[q0:q0 + n].view(n, Hv, dv).float())
            out[q0:q0 + n] = o.reshape(n, Hv * dv).to(out.dtype)
        return out @ L["out"].t()

    def _attn(self, x, L, ai, chunk, arena):
        """Gated full attention; ai = the layer's index among the attention layers (its KV pages)."""
        cfg = self.cfg
        T = x.shape[0]
        QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        kc, vc = arena.layer(ai)
        x = self._q(x)
        qg = (x @ L["wq"].t()).view(T, QH, 2 * D if cfg.attn_output_gate else D)
        q, gate = (qg[..., :D], qg[..., D:]) if cfg.attn_output_gate else (qg, None)
        k = (x @ L["wk"].t()).view(T, KH, D)
        v = (x @ L["wv"].t()).view(T, KH, D)
        rope3 = getattr(chunk, "rope3", None)
        pos = rope3 if rope3 is not None else chunk.positions
        q = rope_partial(rmsnorm_offset(q, L["qn"], cfg.rms_eps), pos, self.cos_sin, cfg.rotary_dim,
                         cfg.mrope_sections)
        k = rope_partial(rmsnorm_offset(k, L["kn"], cfg.rms_eps), pos, self.cos_sin, cfg.rotary_dim,
                         cfg.mrope_sections)
        ok = chunk.slots >= 0
        slots = chunk.slots[ok].long()
        kc.view(-1, KH, D)[slots] = k[ok].to(kc.dtype)
        vc.view(-1, KH, D)[slots] = v[ok].to(vc.dtype)
        o = ref.segmented_attention(q, kc, vc, chunk.seqs, chunk.page_list, self.scale).to(x.dtype)
        if gate is not None:
            o = o.view(T, QH, D) * torch.sigmoid(gate.float())
        return self._q(o.reshape(T, QH * D)) @ L["wo"].t()

    def _q(self, x: torch.Tensor) -> torch.Tensor:
        """Fake-quantize an fp8 GEMM input the way the kernels do (emulation only)."""
        if not self.emulate:
            return x
        from quail_b200.ops.quant import dequantize_mx, quantize_act_mx
        return dequantize_mx(*quantize_act_mx(x.bfloat16().float())).to(x.dtype)

    def _mlp(self, x, wg, wu, wd):
        if self.fp4 and not self.cfg.is_moe:
            from quail_b200.ops.quant import fake_nvfp4_rows
            x4 = fake_nvfp4_rows(x.bfloat16().float())
            gu = torch.cat([x4 @ wg.t(), x4 @ wu.t()], dim=1).bfloat16().float()
            a = ref.silu_mul(gu[:, :wg.shape[0]], gu[:, wg.shape[0]:])
            return fake_nvfp4_rows(a) @ wd.t()
        return self._q(ref.silu_mul(self._q(x) @ wg.t(), self._q(x) @ wu.t())) @ wd.t()

    # ------------------------------------------------------------ forward
    images = None           # engine.images.ImageStore of a model with a vision tower

    @torch.no_grad()
    def hidden_chunk(self, chunk, arena) -> torch.Tensor:
        cfg = self.cfg
        h = image_embeddings(chunk.ids, self.embed, self.images) if cfg.has_vision else self.embed[chunk.ids.long()]
        gi = ai = 0
        for i, L in enumerate(self.layers):
            x = rmsnorm_offset(h, L["ln1"], cfg.rms_eps)
            if cfg.kind(i) == "gdn":
                h = h + self._gdn(x, L, gi, chunk, arena)
                gi += 1
            else:
                h = h + self._attn(x, L, ai, chunk, arena)
                ai += 1
            if self.emulate:
                h = h.bfloat16().float()
            x = rmsnorm_offset(h, L["ln2"], cfg.rms_eps)
            h = h + (self._moe(x, L) if cfg.is_moe else self._mlp(x, L["wg"], L["wu"], L["wd"]))
            if self.emulate:
                h = h.bfloat16().float()
        return h

    def _moe(self, x, L):
        """Routed experts (softmax top-k, renormalized) plus the sigmoid-gated shared expert
        (HF Qwen3_5MoeSparseMoeBlock)."""
        ids, w = ref.moe_route(x @ L["router"].t(), self.cfg.top_k)
        out = torch.zeros_like(x)
        for e in ids.unique().tolist():
            t, j = (ids == e).nonzero(as_tuple=True)
            wg, wu, wd = L["experts"][e]
            out.index_add_(0, t, self._mlp(x[t], wg, wu, wd) * w[t, j, None].to(x.dtype))
        if "shared" in L:
            wg, wu, wd = L["shared"]
            out = out + torch.sigmoid(x @ L["shared_gate"].t()) * self._mlp(x, wg, wu, wd)
        return out

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        h = self.hidden_chunk(chunk, arena)
        if self.cfg.has_sae:
            return ref.sae_features(h[chunk.final_rows.long()], self.sae_w, self.sae_b, self.cfg.sae_keep)
        normed = rmsnorm_offset(h[chunk.final_rows.long()], self.final_norm, self.cfg.rms_eps)
        ans = (normed @ self.answer_rows.t()).float()
        if not getattr(chunk, "full_readout", False):
            return ans
        full = (normed @ self.head.t()).float()
        return ref.head_readout(full, ans, getattr(chunk, "topk", False))
