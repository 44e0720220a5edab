"""Qwen3-MoE decoder (Qwen3-30B-A3B architecture) on the sm_100a kernels.

Attention is Qwen3's (the same kernels as `quail_b200.models.qwen3`); the
MLP of every layer is a softmax router over E experts, top-k with
renormalized weights, and SwiGLU experts. The expert half runs through
`quail_b200.parallel.ep.EPState`: with one rank the dispatch/combine kernels
permute locally, with W ranks (expert parallelism, E / W experts per GPU) they
move token rows over NVLink inside the grouped GEMMs.

Per layer: [x8 = norm(h)] -> QKV GEMM -> qk-norm+RoPE+KV write -> tcgen05
attention -> o GEMM (+residual) -> post-attention norm (e4m3 + bf16) ->
router GEMM -> route/plan/sort -> gate_up (+dispatch, SwiGLU) -> down
(+combine push) -> combine (+residual, next layer's norm).

Reference: the reference loads Qwen3-MoE through vLLM with a fused Triton
MoE (quail/backends/quail/executor/moe.py:12-87, model_loading.py:27-363);
the checkpoint names here are the HF Qwen3-MoE ones (mlp.gate.weight,
mlp.experts.{e}.{gate,up,down}_proj).
"""

from __future__ import annotations

import torch

from quail_b200.models.config import DecoderConfig
from quail_b200.models.weights import head_weight
from quail_b200.ops import reference as ref


def _deq(ckpt, name, device):
    from quail_b200.ops.quant import dequantize_weight
    w = ckpt[name + ".weight"].to(device)
    s = ckpt.get(name + ".weight_scale_inv")
    return w.float() if s is None else dequantize_weight(w, s.to(device))


class Qwen3MoeWeights:
    """Device weights of one rank: attention and router replicated, experts [lo, hi) stacked."""

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor] | None, device, *, experts=None,
                 head_rows=None, seed: int = 0):
        from quail_b200.ops.quant import interleave_gate_up_mx, quantize_weight_mx
        assert cfg.is_moe and cfg.fp8 and cfg.head_dim == 128
        self.cfg = cfg
        self.device = device
        bf = torch.bfloat16
        self.experts = experts if experts is not None else range(cfg.num_experts)
        if ckpt is None:
            ckpt = {}
            self._random = seed
        else:
            self._random = None
        g = self._layer_ckpt(ckpt, "global", device)
        self.embed = g["model.embed_tokens.weight"].to(device=device, dtype=bf).contiguous()
        self.final_norm = g["model.norm.weight"].to(device=device, dtype=bf)
        self.head = head_weight(g, cfg)
        self.layers = []
        for i in range(cfg.layers):
            c = self._layer_ckpt(ckpt, i, device)
            p = f"model.layers.{i}."
            L = {
                "ln1": c[p + "input_layernorm.weight"].to(device=device, dtype=bf),
                "ln2": c[p + "post_attention_layernorm.weight"].to(device=device, dtype=bf),
                "qn": c[p + "self_attn.q_norm.weight"].to(device=device, dtype=bf),
                "kn": c[p + "self_attn.k_norm.weight"].to(device=device, dtype=bf),
                "router": c[p + "mlp.gate.weight"].to(device=device, dtype=bf).contiguous(),
            }
            names = [p + "self_attn.q_proj", p + "self_attn.k_proj", p + "self_attn.v_proj"]
            L["wqkv"], L["sqkv"] = quantize_weight_mx(torch.cat([_deq(c, n, device) for n in names]))
            L["wo"], L["so"] = quantize_weight_mx(_deq(c, p + "self_attn.o_proj", device))
            gu_q, gu_s, d_q, d_s = [], [], [], []
            for e in self.experts:
                q = p + f"mlp.experts.{e}."
                wq, ws = interleave_gate_up_mx(torch.cat([_deq(c, q + "gate_proj", device),
                                                          _deq(c, q + "up_proj", device)]))
                gu_q.append(wq)
                gu_s.append(ws)
                wq, ws = quantize_weight_mx(_deq(c, q + "down_proj", device))
                d_q.append(wq)
                d_s.append(ws)
            # each expert's rows are a multiple of 128, so the stacked scale
            # atoms are the per-expert atoms back to back
            L["wgu"], L["sgu"] = torch.cat(gu_q).contiguous(), torch.cat(gu_s).contiguous()
            L["wd"], L["sd"] = torch.cat(d_q).contiguous(), torch.cat(d_s).contiguous()
            self.layers.append(L)
            del c
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.head_dim, cfg.rope_theta, device=device)
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def _layer_ckpt(self, ckpt, key, device):
        """The checkpoint tensors of one layer (or the global ones): from the
        given dict, or generated from a per-(seed, layer) stream so that every
        rank of an expert-parallel job builds the same replicated weights."""
        if self._random is None:
            return ckpt
        from quail_b200.models.weights import iter_random_layer
        cfg = self.cfg
        gen = torch.Generator(device=device)
        if key == "global":
            gen.manual_seed(self._random * 1_000_003 + 7)
            out = {"model.embed_tokens.weight": (torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=device)
                                                 * cfg.init_std).bfloat16(),
                   "model.norm.weight": torch.ones(cfg.hidden, device=device, dtype=torch.bfloat16)}
            if not cfg.tied_head:
                out["lm_head.weight"] = (torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=device)
                                         * cfg.init_std).bfloat16()
            return out
        out = {}
        gen.manual_seed(self._random * 1_000_003 + 1000 + key)
        for name, t in iter_random_layer(cfg, key, gen, device=device, experts=range(0)):
            out[name] = t
        # experts from their own streams, so a rank generates only its own
        from quail_b200.models.weights import _emit_proj, expert_shapes, layer_prefix
        for e in self.experts:
            eg = torch.Generator(device=device)
            eg.manual_seed(self._random * 1_000_003 + 1_000_000 + key * 4096 + e)
            for name, shape in expert_shapes(cfg).items():
                out.update(_emit_proj(layer_prefix(key) + f"mlp.experts.{e}.{name}", shape, cfg, eg, device,
                                      torch.bfloat16))
        return out

    def head_bf16(self) -> torch.Tensor:
        if getattr(self, "_head_dev", None) is None:
            self._head_dev = self.head.to(device=self.device, dtype=torch.bfloat16).contiguous()
        return self._head_dev

    def set_answer_rows(self, token_ids) -> None:
        ids = torch.as_tensor(list(token_ids), dtype=torch.long)
        self.answer_rows = self.head.index_select(0, ids.to(self.head.device)).to(
            device=self.device, dtype=torch.bfloat16).contiguous()
        self.answer_ids = ids


class Qwen3MoePipeline:
    """Forward pass of a packed chunk: attention on this rank's tokens, experts through EPState."""

    def __init__(self, cfg: DecoderConfig, weights: Qwen3MoeWeights, *, max_tokens: int = 16384, group=None):
        from quail_b200.parallel.ep import EPState
        assert (cfg.num_q_heads // cfg.num_kv_heads) % 4 == 0, "the tcgen05 attention packs 4 q heads per KV head"
        self.cfg = cfg
        self.w = weights
        self.scale = ref.softmax_scale(cfg.head_dim)
        self.ep = EPState(cfg, max_tokens, weights.device, group)
        self.tc_attention = True

    @torch.no_grad()
    def forward_hidden(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        cfg, w = self.cfg, self.w
        h = ops.embed_gather(chunk.ids, w.embed)
        x8, xs = ops.rmsnorm_quant_mx(h, w.layers[0]["ln1"], cfg.rms_eps)
        n = len(w.layers)
        tm = self.ep.timer
        for li, L in enumerate(w.layers):
            kc, vc = arena.layer(li)
            with tm("attention block (qkv, rope, attention, o_proj, norms)"):
                qkv = ops.gemm_mx(x8, xs, L["wqkv"], L["sqkv"])
                q = ops.qk_norm_rope_kv(qkv, chunk.positions, L["qn"], L["kn"], w.cos_sin, chunk.slots, kc, vc,
                                        cfg.num_q_heads, cfg.num_kv_heads, cfg.rms_eps)
                o8, os_ = ops.chunk_attention(q, kc, vc, chunk, self.scale, mx=True, tc=True)
                ops.gemm_mx(o8, os_, L["wo"], L["so"], epi=ops.EPI_RESIDUAL, out=h, residual=h)
                x8, xs = ops.rmsnorm_quant_mx(h, L["ln2"], cfg.rms_eps)
                xb = ops.rmsnorm_quant(h, L["ln2"], cfg.rms_eps, fp8=False)
            nxt = w.layers[li + 1]["ln1"] if li + 1 < n else None
            r = self.ep.forward(x8, xs, xb, h, L, next_norm=nxt, eps=cfg.rms_eps)
            if r is not None:
                x8, xs = r
        return h

    @torch.no_grad()
    def idle_pass(self) -> None:
        """The MoE half of every layer with no tokens of this rank (expert parallelism)."""
        cfg, w = self.cfg, self.w
        h = torch.empty(0, cfg.hidden, dtype=torch.bfloat16, device=w.device)
        e8 = torch.empty(0, cfg.hidden, dtype=torch.float8_e4m3fn, device=w.device)
        esf = torch.empty(0, dtype=torch.uint8, device=w.device)
        for L in w.layers:
            self.ep.forward(e8, esf, h, h, L, next_norm=None, eps=cfg.rms_eps)

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        cfg, w = self.cfg, self.w
        h = self.forward_hidden(chunk, arena)
        if not getattr(chunk, "full_readout", False):
            return ops.final_norm_readout(h, chunk.final_rows, w.final_norm, cfg.rms_eps, w.answer_rows)
        R = chunk.final_rows.numel()
        normed = torch.empty(R, cfg.hidden, dtype=torch.bfloat16, device=h.device)
        ans = ops.final_norm_readout(h, chunk.final_rows, w.final_norm, cfg.rms_eps, w.answer_rows, normed=normed)
        return ops.head_readout(normed, w.head_bf16(), ans, getattr(chunk, "topk", False))
