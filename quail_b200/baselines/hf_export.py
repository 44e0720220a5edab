"""Write a decoder config's weights as a Hugging Face checkpoint directory.

The directory holds `config.json` (Qwen3ForCausalLM), `generation_config.json`
and `model.safetensors` in the names this engine also loads
(quail_b200/models/weights.py): fp8 models keep e4m3 projections with
`weight_scale_inv` 128 x 128 block scales and declare the block-fp8
quantization config, so a stock engine loads exactly the weights this engine
runs. No tokenizer is written: requests carry token ids.
"""

from __future__ import annotations

import json
import os

import torch

from quail_b200.models.config import DecoderConfig


def hf_config(cfg: DecoderConfig) -> dict:
    """The config.json of a dense Qwen3 decoder config."""
    if cfg.arch != "qwen3" or cfg.is_moe or cfg.is_hybrid:
        raise ValueError(f"only dense Qwen3 decoders are exported, not {cfg.name!r}")
    out = {
        "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3",
        "hidden_size": cfg.hidden, "intermediate_size": cfg.intermediate, "num_hidden_layers": cfg.layers,
        "num_attention_heads": cfg.num_q_heads, "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
        "vocab_size": cfg.vocab, "rms_norm_eps": cfg.rms_eps, "rope_theta": cfg.rope_theta,
        "max_position_embeddings": cfg.max_position, "tie_word_embeddings": cfg.tied_head,
        "hidden_act": "silu", "attention_bias": False, "torch_dtype": "bfloat16",
        "bos_token_id": 0, "eos_token_id": 1,
    }
    if cfg.fp8:
        out["quantization_config"] = {"quant_method": "fp8", "activation_scheme": "dynamic",
                                      "fmt": "e4m3", "weight_block_size": [128, 128]}
    return out


def export_checkpoint(cfg: DecoderConfig, out_dir: str, seed: int = 0, device="cpu") -> str:
    """Random-init weights of `cfg` (the same generator as the engine's) into `out_dir`."""
    from safetensors.torch import save_file
    if device == "cpu" or (isinstance(device, torch.device) and device.type == "cpu"):
        from quail_b200.models.weights import random_checkpoint
        ckpt = random_checkpoint(cfg, seed=seed)
    else:
        from quail_b200.models.build import random_checkpoint_on
        ckpt = random_checkpoint_on(cfg, device, seed=seed)
    os.makedirs(out_dir, exist_ok=True)
    tensors = {k: v.detach().to("cpu").contiguous() for k, v in ckpt.items()}
    save_file(tensors, os.path.join(out_dir, "model.safetensors"), metadata={"format": "pt"})
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(hf_config(cfg), f, indent=1)
    with open(os.path.join(out_dir, "generation_config.json"), "w") as f:
        json.dump({"bos_token_id": 0, "eos_token_id": 1, "do_sample": False}, f)
    return out_dir
