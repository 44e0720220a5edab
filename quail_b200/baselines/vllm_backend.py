"""The stock-vLLM request backend: one request per row and call.

A region's calls are answered the way a serving engine answers a client that
sends each row's prompt separately: the whole prompt (instruction prefix,
document, question) is one request of token ids, vLLM's prefix caching shares
what requests have in common, and the answer is read from the log
probabilities of one generated token (filter: the best TRUE spelling against
the best FALSE spelling among the returned candidates; score: sigmoid of that
margin; classify: the label whose first token is likeliest; map: greedy text).
This mirrors the reference's stock baseline (quail/baselines/vllm.py,
request.py, request_scheduling.py): the comparison is the engine, not the
model, so both run the same random-init weights (`hf_export`).
"""

from __future__ import annotations

import math
import tempfile
import time

import numpy as np

from quail_b200.api import prompts as P
from quail_b200.api.engine import RegionOutput

# how many top log probabilities a request returns; answers outside them read as -inf
LOGPROBS = 20
GPU_MEMORY_UTILIZATION = 0.9


def request_tokens(prefix, doc, tail) -> list[int]:
    """One request's prompt token ids: the instruction prefix, the document, the question."""
    return [int(t) for t in np.concatenate([np.asarray(prefix, np.int64), np.asarray(doc, np.int64),
                                            np.asarray(tail, np.int64)])]


def margin_of(logprobs: dict, true_ids, false_ids) -> float:
    """Best TRUE log probability minus best FALSE one among the returned candidates."""
    t = max((logprobs[i] for i in true_ids if i in logprobs), default=-math.inf)
    f = max((logprobs[i] for i in false_ids if i in logprobs), default=-math.inf)
    if t == -math.inf and f == -math.inf:
        return 0.0
    if f == -math.inf:
        return 50.0
    if t == -math.inf:
        return -50.0
    return t - f


class VLLMEngine:
    """A model engine whose regions are answered by vLLM, one request per (row, call)."""

    def __init__(self, config, registry=None, checkpoint_dir: str | None = None):
        from quail_b200.api.config import check_config
        from quail_b200.api.tokenizer import load_tokenizer
        self.config = config
        self.cfg = check_config(config, registry)
        self.tokenizer = load_tokenizer(config.tokenizer or config.weights, self.cfg.vocab)
        path = config.weights or checkpoint_dir
        if path is None:
            from quail_b200.baselines.hf_export import export_checkpoint
            path = export_checkpoint(self.cfg, tempfile.mkdtemp(prefix="qb_vllm_"), seed=config.seed,
                                     device="cuda")
        self.path = path
        self.boot_s = 0.0
        self._llm = None

    def llm(self):
        if self._llm is None:
            from vllm import LLM
            t0 = time.perf_counter()
            self._llm = LLM(model=self.path, skip_tokenizer_init=True, enable_prefix_caching=True,
                            gpu_memory_utilization=GPU_MEMORY_UTILIZATION, max_model_len=8192,
                            seed=self.config.seed, max_logprobs=LOGPROBS)
            self.boot_s = time.perf_counter() - t0
        return self._llm

    def _generate(self, prompts: list[list[int]], max_tokens: int):
        from vllm import SamplingParams, TokensPrompt
        params = SamplingParams(max_tokens=max_tokens, temperature=0.0, logprobs=LOGPROBS, detokenize=False)
        return self.llm().generate([TokensPrompt(prompt_token_ids=p) for p in prompts], params, use_tqdm=False)

    def run_region(self, preamble: str, docs: list, calls: list, *, on_rows=None, stop=None) -> RegionOutput:
        tok = self.tokenizer
        t0 = time.perf_counter()
        prefix = tok.encode(preamble)
        bodies = [tok.encode("" if d is None else d) if not isinstance(d, (list, np.ndarray)) else np.asarray(d)
                  for d in docs]
        true_ids = tok.answer_ids(P.TRUE_SPELLINGS)
        false_ids = tok.answer_ids(P.FALSE_SPELLINGS)
        values = [dict() for _ in docs]
        alive = list(range(len(docs)))
        asked = fresh = 0
        for c in calls:
            if c.guard is not None:
                raise ValueError("the request backend asks every call of every row (no demand guards)")
            tail = tok.encode(c.tail)
            prompts = [request_tokens(prefix, bodies[r], tail) for r in alive]
            gen = 1 if c.kind in ("filter", "score", "classify") else c.max_tokens
            outs = self._generate(prompts, gen)
            asked += len(prompts)
            fresh += sum(len(p) for p in prompts)
            keep = []
            for r, o in zip(alive, outs):
                seq = o.outputs[0]
                first = {k: v.logprob for k, v in (seq.logprobs[0] if seq.logprobs else {}).items()}
                if c.kind in ("filter", "score"):
                    m = margin_of(first, true_ids, false_ids)
                    values[r][c.name] = (m > 0) if c.kind == "filter" else 1.0 / (1.0 + math.exp(-m))
                    if c.kind == "filter" and c.drops and not m > 0:
                        continue
                elif c.kind == "classify":
                    firsts = [int(tok.encode(str(lab))[0]) for lab in c.labels]
                    scores = [first.get(i, -math.inf) for i in firsts]
                    values[r][c.name] = c.labels[int(np.argmax(scores))]
                else:
                    values[r][c.name] = tok.decode(list(seq.token_ids))
                keep.append(r)
            alive = keep
        stats = {"passes": 0, "fresh_tokens": fresh, "documents": len(docs), "rows": len(docs), "asked": asked,
                 "wall_s": time.perf_counter() - t0, "boot_s": self.boot_s, "backend": "vllm"}
        return RegionOutput(values=values, stats=stats)

    def close(self) -> None:
        self._llm = None


def available() -> bool:
    """Whether vLLM's compiled parts load here (a GPU box with the driver)."""
    try:
        import vllm._C  # noqa: F401
        return True
    except Exception:  # noqa: BLE001 - any import failure means no vLLM here
        return False

