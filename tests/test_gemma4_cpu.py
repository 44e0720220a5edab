"""DiffusionGemma's fp32 statement against Hugging Face's Gemma 4 text model, and its chunks.

The statement (quail_b200/models/gemma4.py) runs packed chunks over paged KV:
its logits must equal Hugging Face's Gemma4ForCausalLM on the same random
checkpoint (sliding and global layers, values from the key projection, a
quarter of the global frequency pairs rotated, GeGLU MLP beside the routed
experts, layer scalars, soft-capped tied head). Prompts packed with a shared
prefix, split across chunks, must match the same prompts alone, and a
sliding layer's window must reach into the earlier segments.
Reference: tests/gpu/test_diffusion_gemma_forward.py (forward against the
checkpoint's own implementation) and tests/engine/test_diffusion_gemma.py.
"""

import numpy as np
import pytest
import torch

from quail_b200.engine.arena import KVArena
from quail_b200.engine.stage_executor import StageExecutor, Task
from quail_b200.models import gemma4 as G
from quail_b200.models.config import MODEL_CONFIGS

CFG = MODEL_CONFIGS["diffusion-gemma-tiny"]


@pytest.fixture(scope="module")
def model():
    ckpt = G.random_gemma4(CFG, seed=3, dtype=torch.float32)
    ids = list(range(16))
    return ckpt, G.DiffusionGemmaReference(CFG, ckpt, head_rows=ids)


def _hf(ckpt):
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM
    m = Gemma4ForCausalLM(G.hf_config(CFG)).float().eval()
    sd = {k: v.float() for k, v in ckpt.items() if k != G.SELF_CONDITIONING_NORM}
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected and all(k == "lm_head.weight" for k in missing)
    m.tie_weights()
    return m


def _arena(pages=256, page=16):
    return KVArena.for_model(CFG, pages, page, device="cpu", dtype=torch.float32)


def _alone(model, tokens, full=False):
    arena = _arena()
    ex = StageExecutor(model, arena, 4096)
    got = {}
    ex.submit(Task(key="x", tokens=np.asarray(tokens, dtype=np.int32), pos_start=0, readout=True,
                   full_readout=full, on_done=lambda t, row: got.__setitem__("x", row.float())))
    ex.run()
    return got["x"]


def test_the_arena_keeps_each_layer_geometry():
    a = _arena(8)
    assert a.layer(0)[0].shape[-2:] == (CFG.num_kv_heads, CFG.head_dim)
    assert a.layer(1)[0].shape[-2:] == (CFG.full_kv_heads, CFG.full_head_dim)
    assert a.layer(2)[0].data_ptr() != a.layer(0)[0].data_ptr()


@pytest.mark.parametrize("n", [12, 40])
def test_statement_matches_hugging_face(model, n):
    ckpt, m = model
    hf = _hf(ckpt)
    rng = np.random.default_rng(n)
    toks = rng.integers(0, 4000, n)
    with torch.no_grad():
        logits = hf(torch.as_tensor(toks)[None]).logits[0, -1].float()
    row = _alone(m, toks, full=True)
    want = logits[:16]
    assert torch.allclose(row[:16], want, rtol=1e-4, atol=1e-4), (row[:16] - want).abs().max()
    assert int(row[16]) == int(logits.argmax())                    # the full-vocabulary argmax
    assert float(row[17]) == pytest.approx(float(torch.logsumexp(logits, 0)), rel=1e-5)


@pytest.mark.parametrize("chunk_tokens", [24, 1000])
def test_packed_chunks_match_prompts_alone(model, chunk_tokens):
    _, m = model
    rng = np.random.default_rng(1)
    prefix = rng.integers(0, 1000, 20).astype(np.int32)
    docs = [rng.integers(0, 1000, k).astype(np.int32) for k in (3, 30, 9)]
    suffix = np.concatenate([rng.integers(0, 1000, 5), G.canvas_ids(CFG)]).astype(np.int32)
    arena = _arena()
    ex = StageExecutor(m, arena, chunk_tokens, min_piece=8)
    got = {}
    ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
    for i, d in enumerate(docs):
        ex.submit(Task(key=("d", i), tokens=np.concatenate([d, suffix]), pos_start=len(prefix),
                       reads=[("p", len(prefix))], readout=True,
                       on_done=lambda t, row, i=i: got.__setitem__(i, row.float())))
    ex.run()
    for i, d in enumerate(docs):
        want = _alone(m, np.concatenate([prefix, d, suffix]))
        assert torch.allclose(got[i], want, rtol=1e-4, atol=1e-4), (i, (got[i] - want).abs().max())
    ex.free("p")
    assert arena.pool.free_pages == arena.pool.num_pages


def test_canvas_rows_read_their_embedding_through_the_canvas_norm(model):
    _, m = model
    ids = G.canvas_ids(CFG)
    assert ids.shape == (CFG.canvas_tokens,) and (ids >= G.CANVAS_TOKEN_BASE).all()
    assert (G.canvas_ids(CFG) == ids).all()                       # the same after every question
    tok = torch.as_tensor(np.concatenate([[7], ids]))
    h = G.embed_rows(tok, m.embed, CFG.embed_scale, m.canvas_norm, CFG.rms_eps)
    plain = m.embed[int(ids[0]) - G.CANVAS_TOKEN_BASE] * CFG.embed_scale
    assert torch.allclose(h[1], G.rms(plain[None], m.canvas_norm, CFG.rms_eps)[0])
    assert torch.allclose(h[0], m.embed[7] * CFG.embed_scale)


def test_sliding_window_reaches_into_earlier_segments():
    """A sliding layer's window counts positions across the prefix and document segments."""
    from quail_b200.ops import reference as ref
    torch.manual_seed(0)
    P, KH, D, W = 4, 1, 8, 5
    k = torch.randn(16, P, KH, D)
    v = torch.randn(16, P, KH, D)
    q = torch.randn(3, 1, D)
    # two segments: 6 keys on pages 0-1, then an own segment of 3 on pages 2
    seqs = torch.tensor([[0, 3, 2, 0, 6, 3, 0, 0, 0, 2, 0, 0]], dtype=torch.int32)
    pl = torch.tensor([0, 1, 2], dtype=torch.int32)
    got = ref.segmented_attention(q, k, v, G.window_seqs(seqs, W), pl, 1.0)
    keys = torch.cat([k.reshape(-1, KH, D)[:6], k.reshape(-1, KH, D)[8:11]])[:, 0]
    vals = torch.cat([v.reshape(-1, KH, D)[:6], v.reshape(-1, KH, D)[8:11]])[:, 0]
    for t in range(3):
        pos = 6 + t
        lo = pos - W + 1
        s = q[t, 0] @ keys[lo:pos + 1].t()
        want = torch.softmax(s, 0) @ vals[lo:pos + 1]
        assert torch.allclose(got[t], want, atol=1e-5)
