"""The stock-vLLM comparison backend: checkpoint export, request building, answer reading.

vLLM itself needs a GPU; here the exported checkpoint is checked against an
independent forward (Hugging Face transformers loads it and must give the
logits this engine's fp32 model gives), and the backend's request and answer
logic runs against a stand-in for vLLM's generate.
"""

import math
import types

import numpy as np
import pyarrow as pa
import pytest
import torch

import quail_b200 as quail
from quail_b200.baselines import register_baselines
from quail_b200.baselines.hf_export import export_checkpoint, hf_config
from quail_b200.baselines.vllm_backend import VLLMEngine, margin_of, request_tokens
from quail_b200.extensions import built_in_registry
from quail_b200.models.config import MODEL_CONFIGS, QWEN3_TINY


def test_the_exported_checkpoint_is_the_engines_network(tmp_path):
    from transformers import Qwen3ForCausalLM

    from quail_b200.models.qwen3 import Qwen3Reference
    from quail_b200.models.weights import load_checkpoint, random_checkpoint
    cfg = QWEN3_TINY.with_(vocab=4096)
    out = export_checkpoint(cfg, str(tmp_path / "ckpt"), seed=3)
    back = load_checkpoint(out)
    mine = random_checkpoint(cfg, seed=3)
    assert set(back) == set(mine) and all(torch.equal(back[k], mine[k].to(back[k].dtype)) for k in mine)
    hf = Qwen3ForCausalLM.from_pretrained(out, torch_dtype=torch.float32).eval()
    ids = torch.randint(0, 4096, (1, 37), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        want = hf(input_ids=ids).logits[0, -1]
    # the engine's fp32 model on the same ids (one sequence, causal)
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.stage_executor import StageExecutor, Task
    model = Qwen3Reference(cfg, {k: v.float() for k, v in mine.items()}, head_rows=list(range(4096)))
    arena = KVArena(cfg.layers, 16, 16, cfg.num_kv_heads, cfg.head_dim, device="cpu", dtype=torch.float32)
    ex = StageExecutor(model, arena, 64)
    got = {}
    ex.submit(Task(key="s", tokens=ids[0].numpy().astype(np.int32), pos_start=0, readout=True,
                   on_done=lambda t, row: got.__setitem__("r", torch.as_tensor(row).float())))
    ex.run()
    assert torch.allclose(got["r"][:4096], want, atol=2e-3, rtol=1e-3)


def test_fp8_export_declares_block_quantization():
    c = hf_config(MODEL_CONFIGS["qwen3-4b-fp8"])
    assert c["quantization_config"]["weight_block_size"] == [128, 128] and c["tie_word_embeddings"]
    with pytest.raises(ValueError, match="dense Qwen3"):
        hf_config(MODEL_CONFIGS["qwen3.5-tiny"])


def test_margins_and_requests():
    assert request_tokens([1, 2], np.array([3]), [4, 5]) == [1, 2, 3, 4, 5]
    assert margin_of({7: -0.1, 9: -2.0}, [7], [9]) == pytest.approx(1.9)
    assert margin_of({9: -2.0}, [7], [9]) < 0 and margin_of({}, [7], [9]) == 0.0


class _Out:
    def __init__(self, lp, ids=(5,)):
        self.outputs = [types.SimpleNamespace(logprobs=[{k: types.SimpleNamespace(logprob=v) for k, v in lp.items()}],
                                              token_ids=list(ids))]


def test_sql_through_the_request_backend(tmp_path, monkeypatch):
    reg = built_in_registry()
    register_baselines(reg)
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", backend="vllm", weights=str(tmp_path))
    sent = []

    def fake_generate(self, prompts, max_tokens):
        sent.append((len(prompts), max_tokens))
        tok = self.tokenizer
        t, f = tok.answer_ids(["TRUE"])[0], tok.answer_ids(["FALSE"])[0]
        # rows whose prompt is odd-length answer TRUE
        return [_Out({t: -0.1, f: -3.0} if len(p) % 2 else {t: -3.0, f: -0.1}) for p in prompts]
    monkeypatch.setattr(VLLMEngine, "_generate", fake_generate)
    with quail.Session(config=cfg, registry=reg) as s:
        docs = ["a", "a b", "a b c", "a b c d"]
        s.register("t", quail.DocumentProvider.from_table(pa.table({"id": [0, 1, 2, 3], "body": docs}),
                                                          id_col="id"))
        res = s.sql("SELECT id, AI.SCORE(PROMPT('Is {0} long?', body)) AS p FROM t "
                    "WHERE AI.IF(PROMPT('Is {0} short?', body))").run()
    kept = res.table.column("id").to_pylist()
    assert sent[0] == (4, 1)                       # every row's own request, one token each
    assert sent[1] == (len(kept), 1)               # the projection asks only the kept rows
    assert all(0 < p < 1 for p in res.table.column("p").to_pylist())
    assert res.report["regions"][0]["backend"] == "vllm"
    with pytest.raises(Exception, match="unknown backend"):
        quail.Session(config=quail.EngineConfig(model="qwen3-tiny", device="cpu", backend="vllm"))
