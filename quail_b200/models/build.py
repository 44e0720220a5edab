"""Building a model replica on a GPU from a checkpoint or from random init."""

from __future__ import annotations

import torch

from quail_b200.models.config import DecoderConfig
from quail_b200.models.qwen3 import Qwen3Pipeline, Qwen3Weights
from quail_b200.models.weights import iter_random_layer

# answer-row token ids used by the synthetic configs (TRUE spellings, then FALSE)
SYNTHETIC_TRUE_IDS = (20611, 3007, 2514, 3007 + 1)
SYNTHETIC_FALSE_IDS = (30351, 4049, 4049 + 1, 30351 + 1)


def random_checkpoint_on(cfg: DecoderConfig, device, seed: int = 0) -> dict[str, torch.Tensor]:
    """Random-init weights in checkpoint format, generated layer by layer on `device`."""
    if cfg.gemma4:
        from quail_b200.models.gemma4 import random_gemma4
        return random_gemma4(cfg, seed=seed, device=device, dtype=torch.bfloat16)
    gen = torch.Generator(device=device).manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    out["model.embed_tokens.weight"] = (torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=device)
                                        * cfg.init_std).bfloat16()
    for i in range(cfg.layers):
        out.update(iter_random_layer(cfg, i, gen, device=device, dtype=torch.bfloat16))
    from quail_b200.models.weights import final_norm_name
    out[final_norm_name(cfg)] = (torch.zeros if cfg.norm_offset else torch.ones)(cfg.hidden, device=device,
                                                                                dtype=torch.bfloat16)
    if not cfg.tied_head:
        out["lm_head.weight"] = (torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=device)
                                 * cfg.init_std).bfloat16()
    from quail_b200.models.weights import random_sae
    out.update(random_sae(cfg, gen, device))
    if cfg.has_vision:
        from quail_b200.models.vision import random_vision
        out.update(random_vision(cfg, gen, device))
    if cfg.decision_head:
        from quail_b200.models.decision import random_decision_head
        out.update(random_decision_head(cfg.hidden, cfg.decision_head_dim, gen, device))
    return out


def build_pipeline(cfg: DecoderConfig, device="cuda", seed: int = 0, ckpt=None,
                   answer_ids=SYNTHETIC_TRUE_IDS + SYNTHETIC_FALSE_IDS, max_tokens: int = 16384 + 256):
    if ckpt is None:
        ckpt = random_checkpoint_on(cfg, device, seed)
    if cfg.gemma4:
        from quail_b200.models.gemma4 import DiffusionGemmaPipeline
        pipe = DiffusionGemmaPipeline(cfg, ckpt, device, head_rows=answer_ids, max_tokens=max_tokens)
        del ckpt
        return pipe
    if cfg.is_hybrid:
        if cfg.arch == "lfm2":
            from quail_b200.models.lfm2 import Lfm2Pipeline as Pipe
        else:
            from quail_b200.models.qwen3_5_gpu import Qwen35Pipeline as Pipe
        kw = {"max_tokens": max_tokens} if cfg.is_moe else {}
        pipe = Pipe(cfg, ckpt, device, head_rows=answer_ids, **kw)
        del ckpt
        torch.cuda.empty_cache() if torch.cuda.is_available() else None
        return pipe
    weights = Qwen3Weights(cfg, ckpt, device, head_rows=answer_ids)
    del ckpt
    torch.cuda.empty_cache() if torch.cuda.is_available() else None
    return Qwen3Pipeline(cfg, weights)
