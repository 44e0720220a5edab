"""Image documents: tokens, multimodal rotary positions, and AI calls over images on the CPU model."""

import io

import numpy as np
import pyarrow as pa
import pytest
import torch

import quail_b200 as quail
from quail_b200.engine.images import IMAGE_TOKEN_BASE, ImageStore
from quail_b200.models.config import MODEL_CONFIGS


def _png(w, h, seed=0):
    from PIL import Image
    rgb = np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)
    buf = io.BytesIO()
    Image.fromarray(rgb).save(buf, format="PNG")
    return buf.getvalue()


def test_image_tokens_and_rotary_positions():
    cfg = MODEL_CONFIGS["qwen3.5-vl-tiny"]
    store = ImageStore(cfg, longest=128)
    toks = store.add(_png(96, 64))              # 3 x 2 tokens
    assert toks[0] == cfg.vision_start_id and toks[-1] == cfg.vision_end_id
    assert (toks[1:-1] == IMAGE_TOKEN_BASE + np.arange(6)).all()
    assert (store.add(_png(96, 64)) == toks).all()          # the same bytes: the same image
    # text, start, 6 image tokens, end, text: the image reads (s, s+i, s+j); after it positions
    # advance by max(rows, cols) = 3, not 6
    seq = np.concatenate([[5, 6], toks, [7, 8]])
    r3, shift = store.rope_positions(seq, np.arange(10, 10 + len(seq)), 0)
    assert (r3[:3] == np.arange(10, 13)[:, None]).all()      # text and the start token
    s = 13
    assert r3[3:9].tolist() == [[s, s, s], [s, s, s + 1], [s, s, s + 2], [s, s + 1, s], [s, s + 1, s + 1],
                                [s, s + 1, s + 2]]
    assert r3[9].tolist() == [s + 3] * 3 and shift == 3      # the end token, then text
    # a piece that starts mid-image continues it
    a, sh = store.rope_positions(seq[:5], np.arange(10, 15), 0)
    b, sh2 = store.rope_positions(seq[5:], np.arange(15, 10 + len(seq)), sh)
    assert (np.concatenate([a, b]) == r3).all() and sh2 == 3


def test_ai_calls_over_image_documents():
    cfg = quail.EngineConfig(model="qwen3.5-vl-tiny", device="cpu", extra={"image_longest": 96})
    imgs = [_png(64, 64, 1), _png(96, 32, 2), _png(64, 64, 1)]
    t = pa.table({"id": [0, 1, 2], "img": pa.array(imgs, pa.binary())})
    with quail.Session(config=cfg) as s:
        s.register("pics", quail.DocumentProvider.from_table(t, id_col="id"))
        out = s.sql("SELECT id, AI.SCORE(PROMPT('Is {0} a cat?', AI.IMAGE(img, 96))) AS p FROM pics "
                    "ORDER BY id").collect()
        p = out.column("p").to_pylist()
        assert all(0 < x < 1 for x in p) and p[0] == pytest.approx(p[2])   # the same image, the same answer
        eng = s.engine()
        assert eng.images.next > 0 and eng.executor.packer.rope_shift
    # a text-only model refuses an image document
    with quail.Session(config=quail.EngineConfig(model="qwen3.5-tiny", device="cpu")) as s:
        s.register("pics", quail.DocumentProvider.from_table(t, id_col="id"))
        with pytest.raises(Exception, match="vision tower"):
            s.sql("SELECT AI.IF(PROMPT('Is {0} a cat?', AI.IMAGE(img, 96))) FROM pics").collect()


def test_image_tokens_change_the_answer_by_their_pixels():
    from quail_b200.api.engine import CallSpec, ModelEngine
    eng = ModelEngine(quail.EngineConfig(model="qwen3.5-vl-tiny", device="cpu"))
    call = CallSpec(kind="score", tail="\\nIs it red?\\nANSWER:", name="p")
    a = eng.run_region("DOCUMENT:\\n", [_png(64, 64, 3), _png(64, 64, 4)], [call]).values
    assert a[0]["p"] != a[1]["p"]
    with torch.no_grad():
        assert eng.images.table("cpu", torch.float32).shape == (8, eng.cfg.hidden)
