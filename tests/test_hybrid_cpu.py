"""The Qwen3.5 hybrid (Gated DeltaNet + gated attention) on CPU: state slots,
chunked prefill pieces and borrowed prefixes against each prompt run alone."""

import numpy as np
import pytest
import torch

from quail_b200.engine.arena import KVArena, PagePool
from quail_b200.engine.stage_executor import StageExecutor, Task
from quail_b200.models.config import QWEN35_TINY
from quail_b200.models.qwen3_5 import Qwen35Reference, delta_rule
from quail_b200.models.weights import random_checkpoint


@pytest.fixture(scope="module", params=["qwen3.5-tiny", "qwen3.6-moe-tiny"])
def model(request):
    from quail_b200.models.config import MODEL_CONFIGS
    cfg = MODEL_CONFIGS[request.param].with_(vocab=1000, max_position=4096)
    ckpt = random_checkpoint(cfg, seed=4, dtype=torch.float32)
    return cfg, Qwen35Reference(cfg, ckpt, head_rows=(11, 12, 13, 14))


def test_state_slots_follow_keys_and_borrows():
    pool = PagePool(20, 4, state_slots=3)
    pool.alloc("p", 5)
    pool.alloc("a", 3)
    pool.borrow("a", "p")
    pool.alloc("b", 3)
    assert pool.alloc("c", 1) is None            # no state slot left
    pool.free_key("p")                           # still held by a's borrow
    assert len(pool.slot_free) == 0
    pool.free_key("a")
    assert len(pool.slot_free) == 2 and pool.alloc("c", 1) is not None   # a's slot and its hold on p
    pool.check()
    for k in ("b", "c"):
        pool.free_key(k)
    assert len(pool.slot_free) == 3
    pool.check()


def test_delta_rule_stores_and_recalls():
    """beta = 1, no decay, orthonormal keys: the state maps each key to its value."""
    torch.manual_seed(0)
    dk = dv = 8
    keys = torch.linalg.qr(torch.randn(dk, dk))[0][:3]          # 3 orthonormal keys
    vals = torch.randn(3, dv)
    S = torch.zeros(1, dk, dv)
    k = keys[:, None, :]
    delta_rule(k, k, vals[:, None, :], torch.zeros(3, 1), torch.ones(3, 1), S)
    for i in range(3):
        assert torch.allclose(keys[i] @ S[0], vals[i], atol=1e-5)
    # decay: g = log(0.5) halves the state before the update
    S2 = S.clone()
    out = delta_rule(k[:1], k[:1], vals[:1, None, :], torch.full((1, 1), float(np.log(0.5))), torch.zeros(1, 1), S2)
    assert torch.allclose(S2, 0.5 * S, atol=1e-6) and torch.allclose(out[0, 0], 0.5 * vals[0], atol=1e-5)


def _arena(cfg, pages=400, page=16):
    return KVArena.for_model(cfg, pages, page, device="cpu", dtype=torch.float32, state_slots=48)


def _alone(model, cfg, tokens):
    """One prompt in one sequence of one chunk, nothing borrowed."""
    arena = _arena(cfg)
    ex = StageExecutor(model, arena, 4096)
    got = {}
    ex.submit(Task(key="x", tokens=np.asarray(tokens, dtype=np.int32), pos_start=0, readout=True,
                   on_done=lambda t, row: got.__setitem__("x", row.float())))
    ex.run()
    return got["x"]


@pytest.mark.parametrize("chunk_tokens", [64, 1000])
def test_hybrid_chunks_match_prompts_alone(model, chunk_tokens):
    cfg, m = model
    rng = np.random.default_rng(0)
    prefix = rng.integers(0, 1000, 48).astype(np.int32)
    docs = [rng.integers(0, 1000, n).astype(np.int32) for n in (5, 130, 33, 200)]
    suffix = rng.integers(0, 1000, 7).astype(np.int32)
    arena = _arena(cfg)
    ex = StageExecutor(m, arena, chunk_tokens, min_piece=8)
    got = {}
    ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
    for i, d in enumerate(docs):
        ex.submit(Task(key=("d", i), tokens=np.concatenate([d, suffix]), pos_start=len(prefix),
                       reads=[("p", len(prefix))], readout=True,
                       on_done=lambda t, row, i=i: got.__setitem__(i, row.float())))
    ex.run()
    for i, d in enumerate(docs):
        want = _alone(m, cfg, np.concatenate([prefix, d, suffix]))
        assert torch.allclose(got[i], want, rtol=1e-4, atol=1e-4), (i, (got[i] - want).abs().max())
    ex.free("p")
    assert arena.pool.free_pages == arena.pool.num_pages
    assert len(arena.pool.slot_free) == arena.pool.state_slots
    arena.pool.check()


def test_hybrid_session_filter_and_map():
    import pyarrow as pa

    import quail_b200 as quail
    cfg = quail.EngineConfig(model="qwen3.5-tiny", device="cpu", chunk_tokens=128)
    t = pa.table({"id": [0, 1, 2, 3], "body": ["the plot is long", "great music", "bad ending", "short story"]})
    with quail.Session(config=cfg) as s:
        s.register("r", quail.DocumentProvider.from_table(t, id_col="id"))
        kept = s.sql("SELECT id FROM r WHERE AI.IF(PROMPT('Is it about music? {0}', body))").collect()
        assert set(kept.column("id").to_pylist()) <= {0, 1, 2, 3}
        out = s.sql("SELECT id, AI.MAP(body, 'Summarize', 4) AS m FROM r").collect()
        assert out.num_rows == 4 and all(isinstance(v, str) for v in out.column("m").to_pylist())


@pytest.mark.parametrize("chunk_tokens", [64, 1000])
def test_lfm2_chunks_match_prompts_alone(chunk_tokens):
    from quail_b200.models.config import LFM2_TINY
    from quail_b200.models.lfm2 import Lfm2Reference
    cfg = LFM2_TINY.with_(vocab=1000, max_position=4096)
    m = Lfm2Reference(cfg, random_checkpoint(cfg, seed=6, dtype=torch.float32), head_rows=(1, 2, 3))
    rng = np.random.default_rng(1)
    prefix = rng.integers(0, 1000, 48).astype(np.int32)
    docs = [rng.integers(0, 1000, n).astype(np.int32) for n in (3, 90, 150)]
    suffix = rng.integers(0, 1000, 5).astype(np.int32)
    arena = _arena(cfg)
    ex = StageExecutor(m, arena, chunk_tokens, min_piece=8)
    got = {}
    ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
    for i, d in enumerate(docs):
        ex.submit(Task(key=("d", i), tokens=np.concatenate([d, suffix]), pos_start=len(prefix),
                       reads=[("p", len(prefix))], readout=True,
                       on_done=lambda t, row, i=i: got.__setitem__(i, row.float())))
    ex.run()
    for i, d in enumerate(docs):
        want = _alone(m, cfg, np.concatenate([prefix, d, suffix]))
        assert torch.allclose(got[i], want, rtol=1e-4, atol=1e-4), (i, (got[i] - want).abs().max())


def test_lfm2_session():
    import pyarrow as pa

    import quail_b200 as quail
    cfg = quail.EngineConfig(model="lfm2-tiny", device="cpu", chunk_tokens=128)
    t = pa.table({"id": [0, 1, 2], "body": ["the plot is long", "great music", "bad ending"]})
    with quail.Session(config=cfg) as s:
        s.register("r", quail.DocumentProvider.from_table(t, id_col="id"))
        r = s.sql("SELECT id, AI.SCORE(PROMPT('Is it about music? {0}', body)) AS s FROM r").collect()
        assert r.num_rows == 3 and all(0.0 <= v <= 1.0 for v in r.column("s").to_pylist())


def test_hybrid_sae_features_session():
    import pyarrow as pa

    import quail_b200 as quail
    cfg = quail.EngineConfig(model="qwen3.5-sae-tiny", device="cpu", chunk_tokens=128)
    t = pa.table({"id": [0, 1], "body": ["the plot is long", "great music"]})
    with quail.Session(config=cfg) as s:
        s.register("r", quail.DocumentProvider.from_table(t, id_col="id"))
        r = s.sql("SELECT id, AI.SAE_FEATURES(PROMPT('{0} What is it?', body), {'pooling': 'max'}) AS f FROM r").collect()
        for feats in r.column("f").to_pylist():
            x = [d["strength"] for d in feats]
            assert x == sorted(x, reverse=True) and all(v > 0 for v in x)
