"""Sessions over several GPUs through the product API: data, tensor and expert parallel copies.

Each runs the same SQL as a one-GPU session of the same model (same random
weights) and compares the rows: data-parallel copies must ask each question
once and return the one-GPU rows; a tensor-parallel copy (fused AG->GEMM /
GEMM->RS kernels) and an expert-parallel copy (fused dispatch / combine)
sum in another order, so a row whose yes / no margin is near zero may flip:
nearly all answers must agree. NVLS is off in NCCL here (a rank that dies
while bound to a multicast object can fault its peers).
"""

import os

import numpy as np
import pyarrow as pa
import pytest
import torch

import quail_b200 as quail

pytestmark = pytest.mark.gpu
two_gpus = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                              reason="needs 2 GPUs")


@pytest.fixture(autouse=True)
def _no_nvls(monkeypatch):
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")


def _table(n=96, seed=0):
    rng = np.random.default_rng(seed)
    words = ["refund", "late", "broken", "great", "thanks", "order", "ending", "cast", "plot", "music"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(20, 300)))) for _ in range(n)]
    return pa.table({"id": list(range(n)), "body": bodies})


Q_IF_CLASSIFY = ("SELECT id, AI.CLASSIFY(body, ['praise', 'complaint', 'question', 'other']) AS k FROM t "
                 "WHERE AI.IF(PROMPT('Does the text mention an order? {0}', body)) ORDER BY id")
Q_SCORE = "SELECT id, AI.SCORE(PROMPT('Is the text positive? {0}', body)) AS s FROM t ORDER BY id"


def _run(cfg, sql, table):
    with quail.Session(config=cfg) as s:
        s.register("t", table)
        res = s.sql(sql).run()
    return res.table, res.report


@two_gpus
def test_data_parallel_session_asks_each_question_once_and_returns_the_one_gpu_rows():
    t = _table()
    one, rep1 = _run(quail.EngineConfig(model="qwen3-gpu-tiny-gqa4", device="b200"), Q_IF_CLASSIFY, t)
    two, rep2 = _run(quail.EngineConfig(model="qwen3-gpu-tiny-gqa4", device="b200", gpus=2), Q_IF_CLASSIFY, t)
    assert two.equals(one)
    assert rep2["asked"] == rep1["asked"]
    assert rep2["evaluated_documents"] == rep1["evaluated_documents"] == t.num_rows


@two_gpus
def test_tensor_parallel_session_answers_as_one_gpu():
    t = _table()
    base = dict(model="qwen3-gpu-tiny-gqa4", device="b200", chunk_tokens=4096)
    one, _ = _run(quail.EngineConfig(**base), Q_SCORE, t)
    tp, rep = _run(quail.EngineConfig(**base, gpus=2, parallel="tp"), Q_SCORE, t)
    a, b = np.array(one.column("s").to_pylist()), np.array(tp.column("s").to_pylist())
    assert tp.column("id").to_pylist() == one.column("id").to_pylist()
    assert np.abs(a - b).max() < 0.05, np.abs(a - b).max()
    assert np.corrcoef(a, b)[0, 1] > 0.9
    # the guarded chain: AI.IF then AI.CLASSIFY on the kept rows (the config-4 query shape)
    one_k, _ = _run(quail.EngineConfig(**base), Q_IF_CLASSIFY, t)
    tp_k, _ = _run(quail.EngineConfig(**base, gpus=2, parallel="tp"), Q_IF_CLASSIFY, t)
    kept1, kept2 = set(one_k.column("id").to_pylist()), set(tp_k.column("id").to_pylist())
    assert len(kept1 ^ kept2) <= max(2, len(kept1) // 10)
    k1 = dict(zip(one_k.column("id").to_pylist(), one_k.column("k").to_pylist()))
    k2 = dict(zip(tp_k.column("id").to_pylist(), tp_k.column("k").to_pylist()))
    both = kept1 & kept2
    assert sum(k1[i] == k2[i] for i in both) >= 0.8 * len(both)


@two_gpus
def test_expert_parallel_session_maps_as_one_gpu():
    t = _table(32, seed=3)
    q = "SELECT id, AI.MAP(body, 'Summarize in three words.', 8) AS m FROM t ORDER BY id"
    base = dict(model="qwen3-moe-gpu-tiny", device="b200", chunk_tokens=4096)
    one, _ = _run(quail.EngineConfig(**base), q, t)
    ep, rep = _run(quail.EngineConfig(**base, gpus=2, parallel="ep"), q, t)
    assert ep.column("id").to_pylist() == one.column("id").to_pylist()
    same = sum(x == y for x, y in zip(one.column("m").to_pylist(), ep.column("m").to_pylist()))
    assert same >= 0.8 * t.num_rows, (same, t.num_rows)
    assert rep["evaluated_documents"] == t.num_rows
