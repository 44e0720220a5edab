"""The Qwen3.5 vision tower against the Hugging Face Qwen3_5VisionModel, and image sizing."""

import numpy as np
import pytest
import torch

from quail_b200.models.config import MODEL_CONFIGS
from quail_b200.models.vision import (PREFIX, VisionReference, image_size, patches_of, pixels, random_vision)


def _hf_tower(cfg, w):
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5VisionConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5VisionModel
    vc = Qwen3_5VisionConfig(depth=cfg.vision_depth, hidden_size=cfg.vision_hidden, num_heads=cfg.vision_heads,
                             intermediate_size=cfg.vision_intermediate, out_hidden_size=cfg.hidden,
                             num_position_embeddings=cfg.vision_pos_embeddings, patch_size=cfg.vision_patch,
                             spatial_merge_size=cfg.vision_merge, temporal_patch_size=cfg.vision_temporal)
    vc._attn_implementation = "eager"
    m = Qwen3_5VisionModel(vc).eval()
    sd = {k[len(PREFIX):]: v.float() for k, v in w.items()}
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected and not [k for k in missing if "inv_freq" not in k], (missing, unexpected)
    return m


@pytest.mark.parametrize("rows,cols", [(2, 3), (4, 4), (1, 5)])
def test_the_tower_matches_the_hugging_face_model(rows, cols):
    cfg = MODEL_CONFIGS["qwen3.5-vl-tiny"]
    w = random_vision(cfg, torch.Generator().manual_seed(0), dtype=torch.float32)
    rng = np.random.default_rng(rows * 10 + cols)
    rgb = rng.integers(0, 256, (rows * 32, cols * 32, 3), dtype=np.uint8)
    img = pixels(rgb)
    got = VisionReference(cfg, w).encode([img])[0]
    hf = _hf_tower(cfg, w)
    patches, grid = patches_of(img, cfg)
    with torch.no_grad():
        want = hf(patches, grid_thw=torch.tensor([grid])).pooler_output
    assert got.shape == (rows * cols, cfg.hidden)
    assert torch.allclose(got, want, atol=1e-4, rtol=1e-3)


def test_image_sizing():
    cfg = MODEL_CONFIGS["qwen3.5-vl-tiny"]
    assert image_size(640, 480, 448, cfg) == (14, 10)     # 448 x 336 pixels
    assert image_size(50, 50, 448, cfg) == (2, 2)
    assert image_size(10, 1000, 448, cfg) == (1, 14)
