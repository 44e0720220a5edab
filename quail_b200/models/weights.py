"""Checkpoint format: Hugging Face safetensors with Qwen3 tensor names.

fp8 checkpoints (Qwen/Qwen3-*-FP8) hold each projection as e4m3 `weight`
plus an fp32 `weight_scale_inv` of shape [ceil(N/128), K/128]: the
dequantized weight is weight * scale per 128x128 block. The random-init
generator below writes exactly that format (N(0, std) weights quantized with
block-amax scales), so a synthetic model and a downloaded one load through
the same path. Reference loader: quail/backends/quail/executor/model_loading.py.
"""

from __future__ import annotations

import json
import os
from collections.abc import Iterator

import torch

from quail_b200.models.config import DecoderConfig
from quail_b200.ops.quant import quantize_weight

PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def layer_prefix(i: int) -> str:
    return f"model.layers.{i}."


def projection_shapes(cfg: DecoderConfig) -> dict[str, tuple[int, int]]:
    H = cfg.hidden
    return {
        # with an output gate, q_proj emits [q_h | gate_h] per head
        "self_attn.q_proj": (cfg.q_dim * (2 if cfg.attn_output_gate else 1), H),
        "self_attn.k_proj": (cfg.kv_dim, H),
        "self_attn.v_proj": (cfg.kv_dim, H),
        "self_attn.o_proj": (H, cfg.q_dim),
        "mlp.gate_proj": (cfg.intermediate, H),
        "mlp.up_proj": (cfg.intermediate, H),
        "mlp.down_proj": (H, cfg.intermediate),
    }


def expert_shapes(cfg: DecoderConfig) -> dict[str, tuple[int, int]]:
    H, I = cfg.hidden, cfg.moe_intermediate
    return {"gate_proj": (I, H), "up_proj": (I, H), "down_proj": (H, I)}


def _rand(shape, std, gen, device, dtype=torch.float32):
    return (torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std).to(dtype)


def _emit_proj(name, shape, cfg, gen, device, dtype, fp8: bool | None = None):
    w = _rand(shape, cfg.init_std, gen, device)
    if cfg.fp8 if fp8 is None else fp8:
        q, s = quantize_weight(w)
        return {name + ".weight": q, name + ".weight_scale_inv": s}
    return {name + ".weight": w.to(dtype)}


def gdn_shapes(cfg: DecoderConfig) -> dict[str, tuple[int, int]]:
    """Projections of a Gated DeltaNet layer (HF Qwen3.5 names under linear_attn.)."""
    H = cfg.hidden
    kd, vd = cfg.gdn_key_heads * cfg.gdn_key_dim, cfg.gdn_value_heads * cfg.gdn_value_dim
    return {"linear_attn.in_proj_qkv": (2 * kd + vd, H), "linear_attn.in_proj_z": (vd, H),
            "linear_attn.in_proj_b": (cfg.gdn_value_heads, H), "linear_attn.in_proj_a": (cfg.gdn_value_heads, H),
            "linear_attn.out_proj": (H, vd)}


def iter_random_layer(cfg: DecoderConfig, i: int, gen: torch.Generator, device="cpu",
                      dtype=torch.bfloat16, experts: range | None = None) -> Iterator[tuple[str, torch.Tensor]]:
    """Tensors of layer i in checkpoint names (fp8 projections quantized)."""
    if cfg.arch == "lfm2":
        yield from _iter_lfm2_layer(cfg, i, gen, device, dtype)
        return
    if cfg.arch == "lfm3":
        yield from _iter_lfm3_layer(cfg, i, gen, device, dtype)
        return
    p = layer_prefix(i)
    H = cfg.hidden
    # zero-centered norms (scale 1 + w) start at 0; plain ones at 1
    base = torch.zeros if cfg.norm_offset else torch.ones
    one = base(H, device=device, dtype=dtype)
    yield p + "input_layernorm.weight", one.clone()
    yield p + "post_attention_layernorm.weight", one.clone()
    shapes = projection_shapes(cfg)
    if cfg.kind(i) == "gdn":
        yield from _iter_gdn(cfg, p, gen, device, dtype)
    else:
        yield p + "self_attn.q_norm.weight", base(cfg.head_dim, device=device, dtype=dtype)
        yield p + "self_attn.k_norm.weight", base(cfg.head_dim, device=device, dtype=dtype)
        for name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj"):
            yield from _emit_proj(p + name, shapes[name], cfg, gen, device, dtype).items()
    if cfg.is_moe:
        # router logits ~ N(0, 1) per token: gate weight std 1/sqrt(H) on unit-RMS rows
        yield p + "mlp.gate.weight", _rand((cfg.num_experts, H), H ** -0.5, gen, device, dtype)
        if cfg.shared_intermediate:
            S = cfg.shared_intermediate
            for name, shape in (("gate_proj", (S, H)), ("up_proj", (S, H)), ("down_proj", (H, S))):
                yield from _emit_proj(p + f"mlp.shared_expert.{name}", shape, cfg, gen, device, dtype).items()
            yield p + "mlp.shared_expert_gate.weight", _rand((1, H), H ** -0.5, gen, device, dtype)
        for e in (experts if experts is not None else range(cfg.num_experts)):
            for name, shape in expert_shapes(cfg).items():
                yield from _emit_proj(p + f"mlp.experts.{e}.{name}", shape, cfg, gen, device, dtype).items()
    else:
        for name in ("mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
            yield from _emit_proj(p + name, shapes[name], cfg, gen, device, dtype).items()


def _iter_lfm2_layer(cfg: DecoderConfig, i: int, gen, device, dtype):
    """An LFM2 layer in HF names: operator_norm / ffn_norm, conv.{in_proj, conv, out_proj} or
    self_attn.{q,k,v,out}_proj + q/k_layernorm, feed_forward.w1 (gate), w3 (up), w2 (down)."""
    p = layer_prefix(i)
    H = cfg.hidden
    yield p + "operator_norm.weight", torch.ones(H, device=device, dtype=dtype)
    yield p + "ffn_norm.weight", torch.ones(H, device=device, dtype=dtype)
    if cfg.kind(i) == "conv":
        yield from _emit_proj(p + "conv.in_proj", (3 * H, H), cfg, gen, device, dtype).items()
        yield p + "conv.conv.weight", _rand((H, 1, cfg.conv_width), 0.4, gen, device, dtype)
        yield from _emit_proj(p + "conv.out_proj", (H, H), cfg, gen, device, dtype).items()
    else:
        yield p + "self_attn.q_layernorm.weight", torch.ones(cfg.head_dim, device=device, dtype=dtype)
        yield p + "self_attn.k_layernorm.weight", torch.ones(cfg.head_dim, device=device, dtype=dtype)
        for name, shape in (("q_proj", (cfg.q_dim, H)), ("k_proj", (cfg.kv_dim, H)), ("v_proj", (cfg.kv_dim, H)),
                            ("out_proj", (H, cfg.q_dim))):
            yield from _emit_proj(p + "self_attn." + name, shape, cfg, gen, device, dtype).items()
    for name, shape in (("w1", (cfg.intermediate, H)), ("w3", (cfg.intermediate, H)), ("w2", (H, cfg.intermediate))):
        yield from _emit_proj(p + "feed_forward." + name, shape, cfg, gen, device, dtype).items()


def _iter_lfm3_layer(cfg: DecoderConfig, i: int, gen, device, dtype):
    """An LFM3 layer in HF names: sandwich norms (operator_norm, post_operator_norm, ffn_norm,
    post_ffn_norm), conv.{in_proj, conv, out_proj} or self_attn.{q,k,v,gate,o}_proj + q/k_norm,
    feed_forward.w1 (gate), w3 (up), w2 (down). The post norms start at one like the others."""
    p = layer_prefix(i)
    H = cfg.hidden
    for name in ("operator_norm", "post_operator_norm", "ffn_norm", "post_ffn_norm"):
        yield p + name + ".weight", torch.ones(H, device=device, dtype=dtype)
    if cfg.kind(i) == "conv":
        yield from _emit_proj(p + "conv.in_proj", (3 * H, H), cfg, gen, device, dtype).items()
        yield p + "conv.conv.weight", _rand((H, 1, cfg.conv_width), 0.3, gen, device, dtype)
        yield from _emit_proj(p + "conv.out_proj", (H, H), cfg, gen, device, dtype).items()
    else:
        yield p + "self_attn.q_norm.weight", torch.ones(cfg.head_dim, device=device, dtype=dtype)
        yield p + "self_attn.k_norm.weight", torch.ones(cfg.head_dim, device=device, dtype=dtype)
        for name, shape in (("q_proj", (cfg.q_dim, H)), ("k_proj", (cfg.kv_dim, H)), ("v_proj", (cfg.kv_dim, H)),
                            ("gate_proj", (cfg.num_q_heads, H)), ("o_proj", (H, cfg.q_dim))):
            yield from _emit_proj(p + "self_attn." + name, shape, cfg, gen, device, dtype).items()
    for name, shape in (("w1", (cfg.intermediate, H)), ("w3", (cfg.intermediate, H)), ("w2", (H, cfg.intermediate))):
        yield from _emit_proj(p + "feed_forward." + name, shape, cfg, gen, device, dtype).items()


def _iter_gdn(cfg: DecoderConfig, p: str, gen: torch.Generator, device, dtype):
    """A Gated DeltaNet layer: projections, depthwise conv, decay (A_log, dt_bias), gated-norm weight."""
    Hv = cfg.gdn_value_heads
    for name, shape in gdn_shapes(cfg).items():
        # Gated DeltaNet projections stay bf16 in the fp8 checkpoints (gdn_weight_precision = "bf16")
        yield from _emit_proj(p + name, shape, cfg, gen, device, dtype, fp8=False).items()
    yield p + "linear_attn.conv1d.weight", _rand((cfg.gdn_conv_dim, 1, cfg.conv_width), 0.3, gen, device, dtype)
    # per-head decay rate A in [1, 16] and step dt in [1e-3, 1e-1] (softplus(dt_bias) = dt)
    a = 1.0 + 15.0 * torch.rand(Hv, generator=gen, device=device)
    dt = torch.exp(torch.rand(Hv, generator=gen, device=device) * (torch.log(torch.tensor(0.1)) -
                                                                    torch.log(torch.tensor(1e-3))).item()
                   + torch.log(torch.tensor(1e-3)).item())
    yield p + "linear_attn.A_log", torch.log(a).float()
    yield p + "linear_attn.dt_bias", (dt + torch.log(-torch.expm1(-dt))).float()
    yield p + "linear_attn.norm.weight", torch.ones(cfg.gdn_value_dim, device=device, dtype=dtype)


def random_checkpoint(cfg: DecoderConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                      layers: range | None = None) -> dict[str, torch.Tensor]:
    """A whole random-init checkpoint dict in HF names."""
    if cfg.gemma4:
        from quail_b200.models.gemma4 import random_gemma4
        return random_gemma4(cfg, seed=seed, device=device, dtype=dtype)
    gen = torch.Generator(device=device).manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    out["model.embed_tokens.weight"] = _rand((cfg.vocab, cfg.hidden), cfg.init_std, gen, device, dtype)
    for i in (layers if layers is not None else range(cfg.layers)):
        out.update(iter_random_layer(cfg, i, gen, device, dtype))
    out[final_norm_name(cfg)] = (torch.zeros if cfg.norm_offset else torch.ones)(cfg.hidden, device=device,
                                                                                dtype=dtype)
    if not cfg.tied_head:
        out["lm_head.weight"] = _rand((cfg.vocab, cfg.hidden), cfg.init_std, gen, device, dtype)
    out.update(random_sae(cfg, gen, device))
    if cfg.has_vision:
        from quail_b200.models.vision import random_vision
        out.update(random_vision(cfg, gen, device))
    if cfg.decision_head:
        from quail_b200.models.decision import random_decision_head
        out.update(random_decision_head(cfg.hidden, cfg.decision_head_dim, gen, device))
    return out


def random_sae(cfg: DecoderConfig, gen: torch.Generator, device="cpu") -> dict[str, torch.Tensor]:
    """SAE encoder tensors under `sae.W_enc` [F, H] and `sae.b_enc` [F] (the names of SAE
    checkpoints); empty for a model without one. Encoder rows are unit-norm
    directions scaled to the residual stream's size, the bias a small
    negative threshold, so a row activates a few percent of the features."""
    if not cfg.has_sae:
        return {}
    w = torch.randn(cfg.sae_features, cfg.hidden, generator=gen, device=device, dtype=torch.float32)
    w = w / w.norm(dim=1, keepdim=True) * (0.5 * cfg.hidden ** 0.5)
    b = -0.5 * torch.rand(cfg.sae_features, generator=gen, device=device, dtype=torch.float32)
    return {"sae.W_enc": w.to(torch.bfloat16), "sae.b_enc": b}


def final_norm_name(cfg: DecoderConfig) -> str:
    return "model.embedding_norm.weight" if cfg.arch in ("lfm2", "lfm3") else "model.norm.weight"


def head_weight(ckpt: dict[str, torch.Tensor], cfg: DecoderConfig) -> torch.Tensor:
    return ckpt["model.embed_tokens.weight"] if cfg.tied_head else ckpt["lm_head.weight"]


def save_checkpoint(ckpt: dict[str, torch.Tensor], cfg: DecoderConfig, directory: str) -> None:
    from safetensors.torch import save_file
    os.makedirs(directory, exist_ok=True)
    save_file({k: v.contiguous().cpu() for k, v in ckpt.items()}, os.path.join(directory, "model.safetensors"))
    hf = {
        "architectures": ["Qwen3MoeForCausalLM" if cfg.is_moe else "Qwen3ForCausalLM"],
        "hidden_size": cfg.hidden, "num_hidden_layers": cfg.layers,
        "num_attention_heads": cfg.num_q_heads, "num_key_value_heads": cfg.num_kv_heads,
        "head_dim": cfg.head_dim, "intermediate_size": cfg.intermediate, "vocab_size": cfg.vocab,
        "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.rms_eps, "tie_word_embeddings": cfg.tied_head,
        "max_position_embeddings": cfg.max_position,
    }
    if cfg.is_moe:
        hf.update(num_experts=cfg.num_experts, num_experts_per_tok=cfg.top_k,
                  moe_intermediate_size=cfg.moe_intermediate)
    if cfg.fp8:
        hf["quantization_config"] = {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128],
                                     "activation_scheme": "dynamic"}
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)


def config_from_hf(directory: str, name: str | None = None) -> DecoderConfig:
    with open(os.path.join(directory, "config.json")) as f:
        hf = json.load(f)
    q = hf.get("quantization_config") or {}
    return DecoderConfig(
        name=name or os.path.basename(os.path.normpath(directory)),
        layers=hf["num_hidden_layers"], hidden=hf["hidden_size"], num_q_heads=hf["num_attention_heads"],
        num_kv_heads=hf["num_key_value_heads"], head_dim=hf.get("head_dim", hf["hidden_size"] // hf["num_attention_heads"]),
        intermediate=hf["intermediate_size"], vocab=hf["vocab_size"], rope_theta=hf.get("rope_theta", 1e6),
        rms_eps=hf.get("rms_norm_eps", 1e-6), tied_head=hf.get("tie_word_embeddings", False),
        weight_dtype="fp8" if q.get("quant_method") == "fp8" else "bf16",
        num_experts=hf.get("num_experts", 0), top_k=hf.get("num_experts_per_tok", 0),
        moe_intermediate=hf.get("moe_intermediate_size", 0),
        max_position=hf.get("max_position_embeddings", 40960))


def load_checkpoint(directory: str, device="cpu") -> dict[str, torch.Tensor]:
    """Every safetensors file of a checkpoint directory, by HF tensor name.

    A Decision 2.0 package keeps a bare Qwen3Model (no `model.` prefix) under
    `backbone/` and the head in `decision_head.safetensors`; its backbone
    tensors get the prefix and the head's the `decision_head.` prefix
    (quail/backends/quail/executor/models/decision2_vllm.py:13-25).
    """
    from safetensors.torch import load_file
    out: dict[str, torch.Tensor] = {}
    backbone = os.path.join(directory, "backbone")
    if os.path.isdir(backbone):
        for fn in sorted(os.listdir(backbone)):
            if fn.endswith(".safetensors"):
                for k, v in load_file(os.path.join(backbone, fn), device=str(device)).items():
                    out[k if k.startswith(("model.", "lm_head.")) else "model." + k] = v
        head = os.path.join(directory, "decision_head.safetensors")
        if os.path.exists(head):
            out.update({"decision_head." + k: v for k, v in load_file(head, device=str(device)).items()})
        return out
    for fn in sorted(os.listdir(directory)):
        if fn.endswith(".safetensors"):
            out.update(load_file(os.path.join(directory, fn), device=str(device)))
    return out


def dequantized(ckpt: dict[str, torch.Tensor], name: str) -> torch.Tensor:
    """fp32 value of a projection weight, whatever its stored format: plain, fp8 with
    128x128 block scales (`weight_scale_inv`), or fp8 with per-channel scales
    (`weight_scale`, the FP8-dynamic checkpoints)."""
    w = ckpt[name + ".weight"]
    s = ckpt.get(name + ".weight_scale_inv")
    if s is None:
        pc = ckpt.get(name + ".weight_scale")
        if pc is not None:
            return w.float() * pc.float().reshape(-1, 1).to(w.device)
        return w.float()
    from quail_b200.ops.quant import dequantize_weight
    return dequantize_weight(w, s)
