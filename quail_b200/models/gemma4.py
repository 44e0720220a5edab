"""DiffusionGemma: the Gemma 4 MoE backbone, read in one denoising step at a canvas row.

A filter's or score's prompt ends with a fixed canvas row (a seeded random
vocabulary id, the same after every question); the answer is the TRUE/FALSE
logits at that row. A canvas row's input is its embedding through the
self-conditioning module's output RMSNorm, which is what that module gives
with a zero self-conditioning input (the first denoising step). Canvas rows
are marked in the token stream by CANVAS_TOKEN_BASE + id, so the packer and
the executor need no side table.

A layer (Hugging Face's Gemma4TextDecoderLayer, which tests/test_gemma4_cpu.py
checks this statement against):

  x = RMSNorm(h)                                  input_layernorm
  attention: q/k per-head RMSNorm (weights), v per-head RMSNorm (no weight),
    RoPE; sliding layers read the last `sliding_window` positions with 256-wide
    heads, global layers read everything with 512-wide heads, a quarter of the
    frequency pairs rotated (base 1e6), and their values are the key projection
    (k_eq_v); softmax scale 1
  h = h + RMSNorm(o_proj(attn))                   post_attention_layernorm
  x = RMSNorm(h)                                  pre_feedforward_layernorm
  d = down(gelu_tanh(gate(x)) * up(x))            the dense GeGLU MLP
  MoE layers: d = RMSNorm(d) + RMSNorm(experts(RMSNorm(h)))   (_1, _2, pre_2)
    routed by softmax(proj(RMSNorm(h) * scale / sqrt(H))), top k renormalized,
    times the expert's per_expert_scale
  h = (h + RMSNorm(d)) * layer_scalar             post_feedforward_layernorm

The embeddings are multiplied by sqrt(H); the head is the embedding matrix;
logits are soft-capped (c * tanh(logits / c)).

Reference: quail/backends/quail/executor/models/diffusion_gemma.py:1-231 (the
canvas rows, the layer loop, the folded layer scalars) and
quail/specs/data/models/diffusion-gemma-26b-a4b-fp8.toml (the geometry). The
statement and the GPU pipeline below are this build's own.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from quail_b200.models.config import DecoderConfig
from quail_b200.ops import reference as ref

CANVAS_TOKEN_BASE = 1 << 29
SELF_CONDITIONING_NORM = "self_conditioning.post_norm.weight"
# flags of a sliding layer's sequences (seqs column 3): the window over the whole sequence
WINDOW_ALL = 1 << 24


def canvas_ids(cfg: DecoderConfig) -> np.ndarray:
    """The canvas rows after every question: seeded random vocabulary ids, marked."""
    rng = np.random.default_rng(cfg.canvas_seed)
    return (CANVAS_TOKEN_BASE + rng.integers(0, cfg.vocab, max(cfg.canvas_tokens, 0))).astype(np.int32)


# a first draw whose label distribution has at most this entropy (nats) is kept; others are
# averaged over further draws of the answer canvas
CANVAS_ENTROPY_NATS = 0.1


def answer_canvas(cfg: DecoderConfig, doc: int, draw: int) -> np.ndarray:
    """A classification's answer canvas for document `doc` and draw `draw`, marked: row 0 a
    random vocabulary id (seeded by the canvas seed, the document and the draw), row 1 the turn
    close, the rest padding. Every row is a canvas row; they read each other both ways."""
    ids = np.full(cfg.canvas_answer_rows, cfg.canvas_pad, dtype=np.int64)
    ids[1] = cfg.canvas_turn_close
    ids[0] = np.random.default_rng((cfg.canvas_seed, doc, draw)).integers(0, cfg.vocab)
    return (CANVAS_TOKEN_BASE + ids).astype(np.int32)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


def window_seqs(seqs: torch.Tensor, window: int) -> torch.Tensor:
    """The chunk's sequences as a sliding layer reads them: a window over every segment."""
    out = seqs.clone()
    out[:, 3] |= (window << 8) | WINDOW_ALL
    return out


def rope_table(max_pos: int, head_dim: int, theta: float, pairs: float, device=None) -> torch.Tensor:
    """[max_pos, head_dim] cos | sin halves: the first `pairs` share of the frequency pairs
    rotate at base**(-2i / head_dim), the rest do not (cos 1, sin 0)."""
    half = head_dim // 2
    rot = int(pairs * half)
    inv = torch.zeros(half, dtype=torch.float64)
    inv[:rot] = 1.0 / theta ** (torch.arange(rot, dtype=torch.float64) * 2 / head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None]
    return torch.cat([ang.cos(), ang.sin()], dim=1).to(device=device, dtype=torch.float32)


def layer_prefix(i: int) -> str:
    return f"model.layers.{i}."


def _rand(shape, std, gen, device, dtype):
    return (torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std).to(dtype)


def random_gemma4(cfg: DecoderConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16) -> dict:
    """A random-init checkpoint in Hugging Face's Gemma 4 text names (plus the canvas norm)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    H, std = cfg.hidden, cfg.init_std
    out = {"model.embed_tokens.weight": _rand((cfg.vocab, H), std, gen, device, dtype),
           "model.norm.weight": torch.ones(H, device=device, dtype=dtype),
           SELF_CONDITIONING_NORM: 1.0 + _rand((H,), 0.1, gen, device, dtype)}
    for i in range(cfg.layers):
        p = layer_prefix(i)
        kh, d = cfg.attn_geometry(i)
        full = cfg.kind(i) == "attn"
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            out[p + n + ".weight"] = 1.0 + _rand((H,), 0.1, gen, device, dtype)
        a = p + "self_attn."
        out[a + "q_proj.weight"] = _rand((cfg.num_q_heads * d, H), std, gen, device, dtype)
        out[a + "k_proj.weight"] = _rand((kh * d, H), std, gen, device, dtype)
        if not (full and cfg.k_eq_v):
            out[a + "v_proj.weight"] = _rand((kh * d, H), std, gen, device, dtype)
        out[a + "o_proj.weight"] = _rand((H, cfg.num_q_heads * d), std, gen, device, dtype)
        # the softmax scale is 1: q/k norm weights near d**-0.25 keep q . k near unit variance, as
        # trained checkpoints' small norm weights do (unit weights would make every softmax one-hot)
        qk = d ** -0.25
        out[a + "q_norm.weight"] = qk * (1.0 + _rand((d,), 0.1, gen, device, torch.float32)).to(dtype)
        out[a + "k_norm.weight"] = qk * (1.0 + _rand((d,), 0.1, gen, device, torch.float32)).to(dtype)
        I = cfg.intermediate
        out[p + "mlp.gate_proj.weight"] = _rand((I, H), std, gen, device, dtype)
        out[p + "mlp.up_proj.weight"] = _rand((I, H), std, gen, device, dtype)
        out[p + "mlp.down_proj.weight"] = _rand((H, I), std, gen, device, dtype)
        if cfg.is_moe:
            E, Ie = cfg.num_experts, cfg.moe_intermediate
            out[p + "router.proj.weight"] = _rand((E, H), 1.0, gen, device, dtype)
            out[p + "router.scale"] = 1.0 + _rand((H,), 0.1, gen, device, dtype)
            out[p + "router.per_expert_scale"] = 1.0 + _rand((E,), 0.1, gen, device, dtype)
            out[p + "experts.gate_up_proj"] = _rand((E, 2 * Ie, H), std, gen, device, dtype)
            out[p + "experts.down_proj"] = _rand((E, H, Ie), std, gen, device, dtype)
            for n in ("post_feedforward_layernorm_1", "post_feedforward_layernorm_2", "pre_feedforward_layernorm_2"):
                out[p + n + ".weight"] = 1.0 + _rand((H,), 0.1, gen, device, dtype)
        # layer output scalars sit far below one in trained checkpoints
        out[p + "layer_scalar"] = (0.3 + 0.7 * torch.rand(1, generator=gen, device=device)).to(dtype)
    return out


def rms(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    """Gemma 4's RMSNorm in fp32: x / sqrt(mean(x^2) + eps), times w when given."""
    x = x.float()
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y if w is None else y * w.float()


def rope_rows(x: torch.Tensor, positions: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """NeoX-style rotation of [T, heads, D] by the table's rows at `positions`."""
    half = x.shape[-1] // 2
    cs = table[positions.long()]
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def embed_rows(ids: torch.Tensor, embed: torch.Tensor, scale: float, canvas_norm: torch.Tensor,
               eps: float) -> torch.Tensor:
    """Scaled embeddings; canvas rows (ids >= CANVAS_TOKEN_BASE) through the canvas norm."""
    ids = ids.long()
    canvas = ids >= CANVAS_TOKEN_BASE
    h = embed[torch.where(canvas, ids - CANVAS_TOKEN_BASE, ids)].float() * scale
    if bool(canvas.any()):
        h[canvas] = rms(h[canvas], canvas_norm, eps)
    return h


class DiffusionGemmaReference:
    """fp32 forward over packed chunks (the contract of the other statements: hidden_chunk,
    forward_chunk with answer rows and the full-vocabulary readout)."""

    def __init__(self, cfg: DecoderConfig, ckpt: dict, device="cpu", head_rows=None, dtype=torch.float32):
        assert cfg.gemma4
        self.cfg = cfg
        self.device = device
        f = lambda t: t.to(device=device, dtype=dtype)  # noqa: E731
        self.embed = f(ckpt["model.embed_tokens.weight"])
        self.final_norm = f(ckpt["model.norm.weight"])
        self.canvas_norm = f(ckpt[SELF_CONDITIONING_NORM])
        self.layers = []
        for i in range(cfg.layers):
            p, a = layer_prefix(i), layer_prefix(i) + "self_attn."
            L = {k: f(ckpt[p + n + ".weight"]) for k, n in (
                ("ln_in", "input_layernorm"), ("ln_post_attn", "post_attention_layernorm"),
                ("ln_pre_ffn", "pre_feedforward_layernorm"), ("ln_post_ffn", "post_feedforward_layernorm"))}
            L.update(wq=f(ckpt[a + "q_proj.weight"]), wk=f(ckpt[a + "k_proj.weight"]),
                     wo=f(ckpt[a + "o_proj.weight"]), qn=f(ckpt[a + "q_norm.weight"]),
                     kn=f(ckpt[a + "k_norm.weight"]), wg=f(ckpt[p + "mlp.gate_proj.weight"]),
                     wu=f(ckpt[p + "mlp.up_proj.weight"]), wd=f(ckpt[p + "mlp.down_proj.weight"]),
                     scalar=float(ckpt[p + "layer_scalar"].float().reshape(-1)[0]))
            if a + "v_proj.weight" in ckpt:
                L["wv"] = f(ckpt[a + "v_proj.weight"])
            if cfg.is_moe:
                L.update(wr=f(ckpt[p + "router.proj.weight"]), r_scale=f(ckpt[p + "router.scale"]),
                         r_expert=f(ckpt[p + "router.per_expert_scale"]),
                         egu=f(ckpt[p + "experts.gate_up_proj"]), ed=f(ckpt[p + "experts.down_proj"]))
                for k, n in (("ln_post_ffn1", "post_feedforward_layernorm_1"),
                             ("ln_post_ffn2", "post_feedforward_layernorm_2"),
                             ("ln_pre_ffn2", "pre_feedforward_layernorm_2")):
                    L[k] = f(ckpt[p + n + ".weight"])
            self.layers.append(L)
        self.head = self.embed
        self.rope_swa = rope_table(cfg.max_position, cfg.head_dim, cfg.rope_theta, 1.0, device)
        self.rope_full = rope_table(cfg.max_position, cfg.full_head_dim, cfg.full_rope_theta, cfg.full_rotary_pairs,
                                    device)
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def set_answer_rows(self, token_ids) -> None:
        ids = torch.as_tensor(list(token_ids), dtype=torch.long, device=self.head.device)
        self.answer_rows = self.head.index_select(0, ids)
        self.answer_ids = ids.cpu()

    def _experts(self, x: torch.Tensor, L: dict, h: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        r_in = rms(h, None, cfg.rms_eps) * L["r_scale"].float() * cfg.hidden ** -0.5
        ids, w = ref.moe_route(r_in @ L["wr"].float().t(), cfg.top_k)
        w = w * L["r_expert"].float()[ids]
        out = torch.zeros_like(x)
        Ie = cfg.moe_intermediate
        for e in ids.unique().tolist():
            rows, slot = (ids == e).nonzero(as_tuple=True)
            gu = x[rows] @ L["egu"][e].float().t()
            y = (gelu_tanh(gu[:, :Ie]) * gu[:, Ie:]) @ L["ed"][e].float().t()
            out.index_add_(0, rows, y * w[rows, slot][:, None])
        return out

    @torch.no_grad()
    def hidden_chunk(self, chunk, arena) -> torch.Tensor:
        cfg = self.cfg
        eps = cfg.rms_eps
        T = chunk.ids.shape[0]
        h = embed_rows(chunk.ids, self.embed, cfg.embed_scale, self.canvas_norm, eps)
        seqs_w = window_seqs(chunk.seqs, cfg.sliding_window)
        scale = cfg.attn_scale or ref.softmax_scale(cfg.head_dim)
        ok = chunk.slots >= 0
        slots = chunk.slots[ok].long()
        for i, L in enumerate(self.layers):
            full = cfg.kind(i) == "attn"
            KH, D = cfg.attn_geometry(i)
            QH = cfg.num_q_heads
            table = self.rope_full if full else self.rope_swa
            x = rms(h, L["ln_in"], eps)
            q = rope_rows(rms((x @ L["wq"].float().t()).view(T, QH, D), L["qn"], eps), chunk.positions, table)
            k_raw = (x @ L["wk"].float().t()).view(T, KH, D)
            v_raw = k_raw if "wv" not in L else (x @ L["wv"].float().t()).view(T, KH, D)
            k = rope_rows(rms(k_raw, L["kn"], eps), chunk.positions, table)
            v = rms(v_raw, None, eps)
            kc, vc = arena.layer(i)
            kc.view(-1, KH, D)[slots] = k[ok].to(kc.dtype)
            vc.view(-1, KH, D)[slots] = v[ok].to(vc.dtype)
            o = ref.segmented_attention(q, kc, vc, chunk.seqs if full else seqs_w, chunk.page_list, scale)
            h = h + rms(o @ L["wo"].float().t(), L["ln_post_attn"], eps)
            x = rms(h, L["ln_pre_ffn"], eps)
            d = (gelu_tanh(x @ L["wg"].float().t()) * (x @ L["wu"].float().t())) @ L["wd"].float().t()
            if cfg.is_moe:
                routed = self._experts(rms(h, L["ln_pre_ffn2"], eps), L, h)
                d = rms(d, L["ln_post_ffn1"], eps) + rms(routed, L["ln_post_ffn2"], eps)
            h = (h + rms(d, L["ln_post_ffn"], eps)) * L["scalar"]
        return h

    def _cap(self, logits: torch.Tensor) -> torch.Tensor:
        c = self.cfg.final_softcap
        return c * torch.tanh(logits / c) if c > 0 else logits

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        h = self.hidden_chunk(chunk, arena)
        normed = rms(h[chunk.final_rows.long()], self.final_norm, self.cfg.rms_eps)
        ans = self._cap(normed @ self.answer_rows.float().t())
        if not getattr(chunk, "full_readout", False):
            return ans
        full = self._cap(normed @ self.head.float().t())
        return ref.head_readout(full, ans, getattr(chunk, "topk", False))


def hf_config(cfg: DecoderConfig):
    """Hugging Face's Gemma4TextConfig of `cfg` (for the checks against its model)."""
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    kinds = ["full_attention" if cfg.kind(i) == "attn" else "sliding_attention" for i in range(cfg.layers)]
    return Gemma4TextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
        num_hidden_layers=cfg.layers, num_attention_heads=cfg.num_q_heads, num_key_value_heads=cfg.num_kv_heads,
        head_dim=cfg.head_dim, hidden_activation="gelu_pytorch_tanh", max_position_embeddings=cfg.max_position,
        rms_norm_eps=cfg.rms_eps, tie_word_embeddings=True, sliding_window=cfg.sliding_window, layer_types=kinds,
        final_logit_softcapping=cfg.final_softcap or None, hidden_size_per_layer_input=0,
        num_global_key_value_heads=cfg.full_kv_heads, global_head_dim=cfg.full_head_dim,
        attention_k_eq_v=cfg.k_eq_v, enable_moe_block=cfg.is_moe, num_experts=cfg.num_experts or None,
        top_k_experts=cfg.top_k or None, moe_intermediate_size=cfg.moe_intermediate or None,
        rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": cfg.rope_theta},
                         "full_attention": {"rope_type": "proportional", "rope_theta": cfg.full_rope_theta,
                                            "partial_rotary_factor": cfg.full_rotary_pairs}})


def _pad_rows(w: torch.Tensor, rows: int) -> torch.Tensor:
    return w if w.shape[0] == rows else torch.cat([w, w.new_zeros(rows - w.shape[0], *w.shape[1:])])


def _pad_cols(w: torch.Tensor, cols: int) -> torch.Tensor:
    return w if w.shape[1] == cols else torch.cat([w, w.new_zeros(w.shape[0], cols - w.shape[1])], dim=1)


class DiffusionGemmaPipeline:
    """The forward pass of a packed chunk on the GPU kernels.

    Per layer: RMSNorm kernel -> QKV GEMM (bf16 tcgen05) -> q/k RMSNorm + RoPE + value
    RMSNorm + KV write (one kernel; the global layers' values are the key projection) ->
    small-tile paged attention (head_dim 256 with the sliding window over every segment, or
    512) -> o_proj GEMM -> post-norm residual add fused with the next RMSNorm -> GeGLU MLP (the
    GEMM's GeGLU epilogue, then down) and, in MoE layers, the routed experts on the grouped MX
    GEMMs (GELU gate activation, per-expert scales folded into the down rows) -> the two branch
    norms -> post-norm residual add with the layer scalar folded into its weight.
    Dense widths are padded to multiples of 128 with zero rows (exact: gelu(0) * 0 = 0).
    """

    def __init__(self, cfg: DecoderConfig, ckpt: dict, device, head_rows=None, max_tokens: int = 16384 + 256):
        from quail_b200.ops.quant import interleave_gate_up, interleave_gate_up_mx, quantize_weight_mx
        assert cfg.gemma4
        self.cfg = cfg
        self.device = dev = torch.device(device)
        bf = torch.bfloat16

        def t(name, dtype=bf):
            return ckpt[name].to(device=dev, dtype=dtype).contiguous()
        self.embed = t("model.embed_tokens.weight")
        self.final_norm = t("model.norm.weight")
        self.canvas_norm = t(SELF_CONDITIONING_NORM)
        H = cfg.hidden
        I_pad = -(-cfg.intermediate // 128) * 128
        self.layers = []
        for i in range(cfg.layers):
            p, a = layer_prefix(i), layer_prefix(i) + "self_attn."
            kh, d = cfg.attn_geometry(i)
            full = cfg.kind(i) == "attn"
            scalar = float(ckpt[p + "layer_scalar"].float().reshape(-1)[0])
            L = {"ln_in": t(p + "input_layernorm.weight"), "ln_post_attn": t(p + "post_attention_layernorm.weight"),
                 "ln_pre_ffn": t(p + "pre_feedforward_layernorm.weight"),
                 # the layer scalar multiplies the residual and the branch's norm alike
                 "ln_post_ffn": (ckpt[p + "post_feedforward_layernorm.weight"].float() * scalar).to(dev, bf),
                 "scalar": scalar, "qn": t(a + "q_norm.weight"), "kn": t(a + "k_norm.weight"),
                 "wo": t(a + "o_proj.weight"), "kh": kh, "d": d, "full": full}
            parts = [ckpt[a + "q_proj.weight"], ckpt[a + "k_proj.weight"]]
            L["vmode"] = 2 if a + "v_proj.weight" not in ckpt else 1
            if L["vmode"] == 1:
                parts.append(ckpt[a + "v_proj.weight"])
            L["wqkv"] = torch.cat([w.to(dev, bf) for w in parts]).contiguous()
            g = _pad_rows(ckpt[p + "mlp.gate_proj.weight"].to(dev, torch.float32), I_pad)
            u = _pad_rows(ckpt[p + "mlp.up_proj.weight"].to(dev, torch.float32), I_pad)
            L["wgu"] = interleave_gate_up(torch.cat([g, u]).to(bf)).contiguous()
            L["wd"] = _pad_cols(ckpt[p + "mlp.down_proj.weight"].to(dev, torch.float32), I_pad).to(bf).contiguous()
            if cfg.fp8:
                # fp8 checkpoints: the projections run on the MX (block-scaled e4m3) GEMM
                L["wqkv8"], L["sqkv"] = quantize_weight_mx(L["wqkv"].float())
                L["wo8"], L["so"] = quantize_weight_mx(L["wo"].float())
                L["wgu8"], L["sgu"] = interleave_gate_up_mx(torch.cat([g, u]))
                L["wd8"], L["sd"] = quantize_weight_mx(L["wd"].float())
                for k in ("wqkv", "wo", "wgu", "wd"):
                    del L[k]
            if cfg.is_moe:
                L.update(ln_post_ffn1=t(p + "post_feedforward_layernorm_1.weight"),
                         ln_post_ffn2=t(p + "post_feedforward_layernorm_2.weight"),
                         ln_pre_ffn2=t(p + "pre_feedforward_layernorm_2.weight"),
                         router_in=(ckpt[p + "router.scale"].float() * H ** -0.5).to(dev, bf))
                L["moe"] = self._experts(ckpt, p, interleave_gate_up_mx, quantize_weight_mx)
            self.layers.append(L)
        self.ep = None
        if cfg.is_moe:
            from quail_b200.parallel.ep import EPState
            # the experts always run on the grouped MX (fp8) GEMMs
            self.ep = EPState(cfg.with_(moe_intermediate=self._ie_pad, weight_dtype="fp8"), max_tokens, dev, None)
        self.rope_swa = rope_table(cfg.max_position, cfg.head_dim, cfg.rope_theta, 1.0, dev)
        self.rope_full = rope_table(cfg.max_position, cfg.full_head_dim, cfg.full_rope_theta, cfg.full_rotary_pairs,
                                    dev)
        self.scale = cfg.attn_scale or ref.softmax_scale(cfg.head_dim)
        self.head = self.embed
        self.answer_rows = None
        if head_rows is not None:
            self.set_answer_rows(head_rows)

    def _experts(self, ckpt, p, interleave_gate_up_mx, quantize_weight_mx) -> dict:
        """Router (bf16) and the experts in the grouped GEMMs' MX layout: the expert width padded
        to a multiple of 128, each expert's per_expert_scale folded into its down rows."""
        cfg, dev = self.cfg, self.device
        Ie = cfg.moe_intermediate
        self._ie_pad = -(-Ie // 128) * 128
        gu = ckpt[p + "experts.gate_up_proj"].to(dev, torch.float32)
        down = ckpt[p + "experts.down_proj"].to(dev, torch.float32)
        s = ckpt[p + "router.per_expert_scale"].to(dev, torch.float32)
        gq, gs, dq, ds = [], [], [], []
        for e in range(cfg.num_experts):
            g = _pad_rows(gu[e, :Ie], self._ie_pad)
            u = _pad_rows(gu[e, Ie:], self._ie_pad)
            q, sc = interleave_gate_up_mx(torch.cat([g, u]))
            gq.append(q)
            gs.append(sc)
            q, sc = quantize_weight_mx(_pad_cols(down[e] * s[e], self._ie_pad))
            dq.append(q)
            ds.append(sc)
        return {"router": ckpt[p + "router.proj.weight"].to(dev, torch.bfloat16).contiguous(),
                "wgu": torch.cat(gq).contiguous(), "sgu": torch.cat(gs).contiguous(),
                "wd": torch.cat(dq).contiguous(), "sd": torch.cat(ds).contiguous()}

    def set_answer_rows(self, token_ids) -> None:
        ids = torch.as_tensor(list(token_ids), dtype=torch.long)
        self.answer_rows = self.head.index_select(0, ids.to(self.head.device)).contiguous()
        self.answer_ids = ids

    def head_bf16(self) -> torch.Tensor:
        return self.head

    @torch.no_grad()
    def forward_hidden(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        C = ops.native()
        cfg, dev = self.cfg, self.device
        eps = cfg.rms_eps
        T = chunk.num_tokens
        ids = chunk.ids
        canvas = ids >= CANVAS_TOKEN_BASE
        h = ops.embed_gather(torch.where(canvas, ids - CANVAS_TOKEN_BASE, ids), self.embed)
        h.mul_(cfg.embed_scale)
        h = torch.where(canvas[:, None], ops.rmsnorm_quant(h, self.canvas_norm, eps, fp8=False), h)
        seqs_w = window_seqs(chunk.seqs, cfg.sliding_window)
        x = ops.rmsnorm_quant(h, self.layers[0]["ln_in"], eps, fp8=False)
        for i, L in enumerate(self.layers):
            kh, d = L["kh"], L["d"]
            QH = cfg.num_q_heads
            mx = "wqkv8" in L
            if mx:
                x8, xs = ops.quant_rows_mx(x)
                p = ops.gemm_mx(x8, xs, L["wqkv8"], L["sqkv"])
            else:
                p = ops.gemm(x, L["wqkv"])
            kc, vc = arena.layer(i)
            q = torch.empty(T, QH, d, dtype=torch.bfloat16, device=dev)
            ops.count_launch(1)
            C.qkv_norm_rope_kv(p, QH, kh, chunk.positions, L["qn"], L["kn"],
                               self.rope_full if L["full"] else self.rope_swa, chunk.slots, kc, vc, q, eps, L["vmode"])
            o = torch.empty(T, QH * d, dtype=torch.bfloat16, device=dev)
            ops.small_attention(q, kc, vc, chunk.seqs if L["full"] else seqs_w, chunk.tiles, chunk.dseqs,
                                chunk.page_list, self.scale, o, None, 0)
            if mx:
                o8, os_ = ops.quant_rows_mx(o)
                a = ops.gemm_mx(o8, os_, L["wo8"], L["so"])
            else:
                a = ops.gemm(o, L["wo"])
            x = ops.post_norm_add_norm(a, h, L["ln_post_attn"], L["ln_pre_ffn"], eps)
            if mx:
                x8, xs = ops.quant_rows_mx(x)
                g8, gs = ops.gemm_mx(x8, xs, L["wgu8"], L["sgu"], epi=ops.EPI_GEGLU_FP8)
                dense = ops.gemm_mx(g8, gs, L["wd8"], L["sd"])
            else:
                dense = ops.gemm(ops.gemm(x, L["wgu"], epi=ops.EPI_GEGLU_BF16), L["wd"])
            if cfg.is_moe:
                xb = ops.rmsnorm_quant(h, L["router_in"], eps, fp8=False)
                x8, xs = ops.rmsnorm_quant_mx(h, L["ln_pre_ffn2"], eps)
                routed = torch.zeros_like(h)
                self.ep.forward(x8, xs, xb, routed, L["moe"], next_norm=None, eps=eps)
                both = torch.zeros_like(h)
                ops.post_norm_add_norm(dense, both, L["ln_post_ffn1"], None, eps)
                ops.post_norm_add_norm(routed, both, L["ln_post_ffn2"], None, eps)
                dense = both
            h.mul_(L["scalar"])
            nxt = self.layers[i + 1]["ln_in"] if i + 1 < len(self.layers) else None
            x = ops.post_norm_add_norm(dense, h, L["ln_post_ffn"], nxt, eps)
        return h

    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        cfg = self.cfg
        if getattr(chunk, "full_readout", False):
            raise ValueError("a canvas model answers at its canvas row; it does not decode")
        h = self.forward_hidden(chunk, arena)
        ans = ops.final_norm_readout(h, chunk.final_rows, self.final_norm, cfg.rms_eps, self.answer_rows)
        c = cfg.final_softcap
        return c * torch.tanh(ans / c) if c > 0 else ans
