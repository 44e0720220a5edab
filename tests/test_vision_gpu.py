"""The vision tower on the kernels, multimodal RoPE in the rope kernel, and image documents on the GPU."""

import io

import numpy as np
import pytest
import torch

from quail_b200 import ops
from quail_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp(min=1e-12)).item()


@pytest.fixture(autouse=True)
def _no_kernel_errors():
    torch.manual_seed(0)
    yield
    assert ops.read_and_clear_error(0) == 0


def test_multimodal_rope_in_the_rope_kernel():
    T, QH, KH, D, rd = 37, 4, 2, 256, 64
    proj = torch.randn(T, QH * D + 2 * KH * D, device=DEV).bfloat16()
    pos3 = torch.randint(0, 4000, (T, 3), dtype=torch.int32, device=DEV)
    qw = (0.1 * torch.randn(D, device=DEV)).bfloat16()
    kw = (0.1 * torch.randn(D, device=DEV)).bfloat16()
    cs = ref.rope_cos_sin(8192, rd, 1e7, device=DEV)
    kc = torch.zeros(8, 16, KH, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(128, device=DEV)[:T].int()
    q = torch.empty(T, QH, D, dtype=torch.bfloat16, device=DEV)
    ops.native().hybrid_qk_rope_kv(proj, QH, KH, False, pos3, qw, kw, True, cs, slots, kc, vc, q, 1e-6, 11, 10)
    from quail_b200.models.qwen3_5 import rmsnorm_offset, rope_partial
    want = rope_partial(rmsnorm_offset(proj[:, :QH * D].float().view(T, QH, D), qw, 1e-6), pos3, cs, rd, (11, 11, 10))
    assert rel_err(q, want) < 1e-2


def test_vision_tower_on_the_kernels():
    from quail_b200.models.build import random_checkpoint_on
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.models.vision import VisionPipeline, VisionReference, pixels
    cfg = MODEL_CONFIGS["qwen3.5-vl-gpu-tiny"]
    ckpt = random_checkpoint_on(cfg, DEV, seed=1)
    rng = np.random.default_rng(0)
    imgs = [pixels(rng.integers(0, 256, (h * 32, w * 32, 3), dtype=np.uint8)) for h, w in ((3, 5), (8, 8), (1, 1))]
    got = VisionPipeline(cfg, ckpt, DEV).encode(imgs)
    want = VisionReference(cfg, ckpt, device=DEV).encode(imgs)
    for g, w in zip(got, want):
        assert g.shape == w.shape and rel_err(g, w) < 2e-2


def _png(w, h, seed):
    from PIL import Image
    buf = io.BytesIO()
    Image.fromarray(np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)).save(buf, "PNG")
    return buf.getvalue()


def test_image_documents_on_the_kernels_match_the_fp32_model():
    import quail_b200 as quail
    from quail_b200.api.engine import CallSpec, ModelEngine
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.build import random_checkpoint_on
    from quail_b200.models.qwen3_5 import Qwen35Reference
    from quail_b200.models.vision import VisionReference
    cfg = quail.EngineConfig(model="qwen3.5-vl-gpu-tiny", device="b200", chunk_tokens=2048)
    eng = ModelEngine(cfg)
    docs = [_png(w, h, s) for s, (w, h) in enumerate([(64, 96), (256, 128), (32, 32), (160, 96)] * 3)]
    call = CallSpec(kind="score", tail="\nIs it a photo?\nANSWER:", name="p")
    got = np.array([v["p"] for v in eng.run_region("DOCUMENT:\n", docs, [call]).values])
    m = eng.cfg
    ckpt = random_checkpoint_on(m, eng.device, seed=0)
    exact = Qwen35Reference(m, ckpt, device=eng.device)
    arena = KVArena.for_model(m, 2048, 16, device=eng.device, dtype=torch.float32, state_slots=64)
    ref_eng = ModelEngine.from_replica(cfg, exact, arena, tokenizer=eng.tokenizer)
    ref_eng.images, ref_eng.vision = type(eng.images)(m), VisionReference(m, ckpt, device=eng.device)
    exact.images = ref_eng.images
    ref_eng.executor.packer.images = ref_eng.images
    want = np.array([v["p"] for v in ref_eng.run_region("DOCUMENT:\n", docs, [call]).values])
    da, db = np.log(got / (1 - got)), np.log(want / (1 - want))
    spread = db.max() - db.min()
    assert spread > 1e-3
    assert np.abs(da - db).max() < 0.35 * spread and np.corrcoef(da, db)[0, 1] > 0.9, (da, db)
