"""The model engine behind a session: one model replica per GPU.

`ModelEngine` owns a model replica, its paged KV arena and a stage executor,
and runs *regions*: one table's documents with a chain of AI calls. It
tokenizes the prompt pieces, deduplicates identical documents (each is read
once), retains the LM-head rows every call reads (TRUE/FALSE spellings and
label tokens), runs the chain and turns readouts into SQL values.

device="b200" runs the sm_100a kernel pipeline on the current GPU;
device="cpu" runs the fp32 PyTorch statement of the same model (the CPU
plumbing configuration of the benchmark). With gpus > 1 the session hands
each replica a shard of the documents (`quail_b200.runtime.workers`).

Reference: quail/backends/quail/worker.py (LoadedGpu: load weights, size
the arena, bind answer rows), executor/runtime.py and executor/region.py.
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from quail_b200.api import prompts as P
from quail_b200.api.config import EngineConfig, check_config
from quail_b200.api.tokenizer import load_tokenizer


@dataclass
class CallSpec:
    """One AI call as text: what follows the document, and how to read the answer."""

    kind: str                 # filter | score | classify | map | extract
    tail: str                 # text after the document (question block + answer cue + turn suffix)
    name: str
    labels: list = field(default_factory=list)
    max_tokens: int = 256
    probabilities: bool = False
    pooling: str = "last"     # features: "last" or "max"
    segments: list | None = None   # tail tokenized piece by piece (decision prompts); joins to `tail`
    read: list = field(default_factory=list)   # segments whose last token the decision head reads
    letters: list = field(default_factory=list)  # lettered prompts: option i's answer letter (slot_lm)
    drops: bool = True        # filter: FALSE drops the row from the region (WHERE); else a value only
    # demand guard (quail_b200.sql.guards): the call is asked on an input row only where
    # this formula is TRUE; its `ai` leaves name earlier calls of the same list
    guard: dict | None = None
    # map: decide(text so far) -> "true" | "not_true" | "undecided" for the WHERE test of the
    # answer alone (quail_b200.sql.partial); the answer stops once it is decided NOT TRUE, or
    # decided TRUE when `stop_when_true` (nothing else reads the answer)
    stop: object = None
    stop_when_true: bool = False


@dataclass
class RegionOutput:
    values: list              # per input row: dict call name -> value
    stats: dict


class ModelEngine:
    @classmethod
    def from_replica(cls, config: EngineConfig, model, arena, tokenizer=None) -> "ModelEngine":
        """An engine around an already built model replica and arena (benchmarks, workers)."""
        from quail_b200.engine.stage_executor import StageExecutor
        from quail_b200.planner.budgets import Budgets
        self = cls.__new__(cls)
        self.config = config
        self.cfg = check_config(config)
        self.on_gpu = config.device != "cpu"
        self.device = arena.device
        self.tokenizer = tokenizer or load_tokenizer(config.tokenizer, self.cfg.vocab)
        self.budgets = Budgets.for_model(self.cfg, config.device, gpus=1)
        self.chunk_tokens = config.chunk_tokens or self.budgets.chunk_tokens
        self.model = model
        self.arena = arena
        self.executor = StageExecutor(model, arena, self.chunk_tokens, gpu_timing=config.gpu_timing,
                                      attention=self._attention_path())
        self.retention = bool(config.extra.get("retention", True))
        self._retained_keys = set()
        return self

    def __init__(self, config: EngineConfig, device_index: int = 0, pages: int | None = None, registry=None):
        self.config = config
        self.cfg = check_config(config, registry)
        self.on_gpu = config.device != "cpu"
        if self.on_gpu:
            if not torch.cuda.is_available():
                raise RuntimeError(f"device {config.device!r} needs a CUDA GPU; use device='cpu' to run on the host")
            self.device = torch.device("cuda", device_index)
            torch.cuda.set_device(self.device)
        else:
            self.device = torch.device("cpu")
        self.tokenizer = load_tokenizer(config.tokenizer or config.weights, self.cfg.vocab)
        from quail_b200.planner.budgets import Budgets
        self.budgets = Budgets.for_model(self.cfg, config.device, gpus=1)
        self.chunk_tokens = config.chunk_tokens or self.budgets.chunk_tokens
        # keep finished documents' KV for later regions (evicted first under memory pressure)
        self.retention = bool(config.extra.get("retention", True))
        self._retained_keys = set()
        self._build(pages)

    # ------------------------------------------------------------ model
    def _checkpoint(self):
        from quail_b200.models.weights import load_checkpoint, random_checkpoint
        if self.config.weights:
            return load_checkpoint(self.config.weights, device=self.device)
        if self.on_gpu:
            from quail_b200.models.build import random_checkpoint_on
            return random_checkpoint_on(self.cfg, self.device, seed=self.config.seed)
        return random_checkpoint(self.cfg, seed=self.config.seed, dtype=torch.float32)

    def _attach_head(self, ckpt) -> None:
        """A decision model's option-scoring head, kept in fp32 beside the backbone."""
        if self.cfg.decision_head:
            from quail_b200.models.decision import DecisionHead, head_tensors
            self.model.decision = DecisionHead(head_tensors(ckpt), self.device)

    images = None       # engine.images.ImageStore of a model with a vision tower
    vision = None       # its vision tower (models/vision.py)

    def _attach_vision(self, ckpt) -> None:
        """A Qwen3.5 model's vision tower and the store of its regions' images."""
        if not self.cfg.has_vision:
            return
        from quail_b200.engine.images import ImageStore
        if self.on_gpu:
            from quail_b200.models.vision import VisionPipeline
            self.vision = VisionPipeline(self.cfg, ckpt, self.device)
        else:
            from quail_b200.models.vision import VisionReference
            self.vision = VisionReference(self.cfg, ckpt, device="cpu")
        self.images = ImageStore(self.cfg, int(self.config.extra.get("image_longest", 1024)))
        self.model.images = self.images

    def _build(self, pages: int | None):
        from quail_b200.engine.arena import KVArena
        from quail_b200.engine.stage_executor import StageExecutor
        if self.cfg.set_attention:
            # set attention (LFM3 / d1): whole passes with no KV kept; the pipeline holds
            # its own scratch pages
            from quail_b200.models.lfm3 import Lfm3Pipeline, Lfm3Reference
            ckpt = self._checkpoint()
            if self.on_gpu:
                self.model = Lfm3Pipeline(self.cfg, ckpt, self.device, max_tokens=self.chunk_tokens)
            else:
                self.model = Lfm3Reference(self.cfg, ckpt, device="cpu")
            del ckpt
            self.arena = None
            self.executor = None
            return
        if self.cfg.gemma4:
            # DiffusionGemma: KV pages in two geometries (sliding and global layers), the routed
            # experts on the grouped MX GEMMs; answers at the canvas row after each question
            from quail_b200.models.gemma4 import DiffusionGemmaPipeline, DiffusionGemmaReference
            ckpt = self._checkpoint()
            if self.on_gpu:
                self.model = DiffusionGemmaPipeline(self.cfg, ckpt, self.device, max_tokens=self.chunk_tokens + 256)
                page_tokens, dtype = 128, torch.bfloat16
            else:
                self.model = DiffusionGemmaReference(self.cfg, ckpt, device="cpu")
                page_tokens, dtype = 16, torch.float32
            del ckpt
            n_pages = pages or self.budgets.arena_pages(page_tokens)
            self.arena = KVArena.for_model(self.cfg, n_pages, page_tokens, device=self.device, dtype=dtype)
            self.executor = StageExecutor(self.model, self.arena, self.chunk_tokens,
                                          gpu_timing=self.config.gpu_timing, attention="unified")
            return
        if self.cfg.is_moe and not self.cfg.is_hybrid:
            self._build_moe(pages)
            return
        ckpt = self._checkpoint()
        if self.cfg.is_hybrid:
            if self.cfg.arch == "lfm2":
                from quail_b200.models.lfm2 import Lfm2Pipeline as GpuModel, Lfm2Reference as CpuModel
            else:
                from quail_b200.models.qwen3_5 import Qwen35Reference as CpuModel
                from quail_b200.models.qwen3_5_gpu import Qwen35Pipeline as GpuModel
            if self.on_gpu:
                kw = {"max_tokens": self.chunk_tokens + 256} if self.cfg.is_moe else {}
                self.model = GpuModel(self.cfg, ckpt, self.device, **kw)
                page_tokens, dtype = 128, torch.bfloat16
            else:
                self.model = CpuModel(self.cfg, ckpt, device="cpu")
                page_tokens, dtype = 16, torch.float32
            self._attach_head(ckpt)
            self._attach_vision(ckpt)
            del ckpt
            n_pages = pages or self.budgets.arena_pages(page_tokens)
            self.arena = KVArena.for_model(self.cfg, n_pages, page_tokens, device=self.device, dtype=dtype,
                                           state_slots=self.budgets.state_slots(self.cfg))
            self.executor = StageExecutor(self.model, self.arena, self.chunk_tokens,
                                          gpu_timing=self.config.gpu_timing, attention=self._attention_path())
            if self.images is not None:
                self.executor.packer.images = self.images
            elif self.on_gpu and getattr(self.model, "ep", None) is None and os.environ.get("QB_GRAPHS", "1") != "0":
                # the token mixers' decode step reads its state slots from device metadata, so a
                # decode pass of a hybrid is one graph too (not with images: their rotary positions
                # are host-computed per pass; not with routed experts: their plan syncs the host)
                self.executor.enable_graphs()
            return
        if self.on_gpu:
            from quail_b200.models.qwen3 import Qwen3Pipeline, Qwen3Weights
            self.model = Qwen3Pipeline(self.cfg, Qwen3Weights(self.cfg, ckpt, self.device))
            page_tokens, dtype = 128, torch.bfloat16
        else:
            from quail_b200.models.qwen3 import Qwen3Reference
            self.model = Qwen3Reference(self.cfg, ckpt, device="cpu")
            page_tokens, dtype = 16, torch.float32
        self._attach_head(ckpt)
        del ckpt
        n_pages = pages or self.budgets.arena_pages(page_tokens)
        self.arena = KVArena(self.cfg.layers, n_pages, page_tokens, self.cfg.num_kv_heads, self.cfg.head_dim,
                             device=self.device, dtype=dtype)
        self.executor = StageExecutor(self.model, self.arena, self.chunk_tokens,
                                      gpu_timing=self.config.gpu_timing, attention=self._attention_path())
        if self.on_gpu and os.environ.get("QB_GRAPHS", "1") != "0":
            # decode passes (AI.MAP / AI.EXTRACT steps) replay captured CUDA graphs
            self.executor.enable_graphs()

    def _build_moe(self, pages: int | None):
        """A Qwen3-MoE copy on this GPU (all experts): the routed-expert kernels of the
        expert-parallel path with local buffers; 16-token KV pages (decode-heavy AI.MAP)."""
        from quail_b200.api.config import Refusal, RefusalError
        from quail_b200.engine.arena import KVArena
        from quail_b200.engine.stage_executor import StageExecutor
        from quail_b200.models.qwen3_moe import Qwen3MoePipeline, Qwen3MoeWeights
        if not self.on_gpu:
            raise RefusalError(Refusal(reasons=(f"{self.cfg.name} runs on the GPU kernels only",),
                                       constraint="unsupported_backend_configuration"))
        ckpt = None
        if self.config.weights:
            from quail_b200.models.weights import load_checkpoint
            ckpt = load_checkpoint(self.config.weights, device=self.device)
        weights = Qwen3MoeWeights(self.cfg, ckpt, self.device, head_rows=range(8), seed=self.config.seed)
        del ckpt
        self.model = Qwen3MoePipeline(self.cfg, weights, max_tokens=self.chunk_tokens + 256)
        torch.cuda.empty_cache()
        page_tokens = int(self.config.extra.get("page_tokens", 16))
        if pages is None:
            free, _ = torch.cuda.mem_get_info(self.device)
            per_page = self.cfg.layers * 2 * page_tokens * self.cfg.num_kv_heads * self.cfg.head_dim * 2
            pages = max(64, int(free * 0.7) // per_page)
        self.arena = KVArena(self.cfg.layers, pages, page_tokens, self.cfg.num_kv_heads, self.cfg.head_dim,
                             device=self.device)
        self.executor = StageExecutor(self.model, self.arena, self.chunk_tokens, gpu_timing=self.config.gpu_timing)

    # ------------------------------------------------------------ metrics
    def _snapshot(self) -> dict:
        """Executor counters at a region's start (its metrics are the differences)."""
        st = self.executor.stats
        if self.on_gpu:
            torch.cuda.reset_peak_memory_stats(self.device)
        return {"passes": st.passes, "tokens": st.tokens, "cached": st.cached, "reused": st.reused,
                "replays": st.replays, "evictions": st.evictions, "gpu_ms": st.gpu_ms, "t": time.perf_counter()}

    def _metrics(self, snap: dict, documents: int, rows: int, asked: int, **extra) -> dict:
        """A region's measured metrics: the reference's per-node set (crates/quail/src/report.rs:24-39;
        every count adds across workers, peak_gpu_bytes takes the largest)."""
        st = self.executor.stats
        hits = st.reused - snap["reused"]
        out = {"passes": st.passes - snap["passes"], "fresh_tokens": st.tokens - snap["tokens"],
               "documents": documents, "rows": rows, "asked": asked,
               "wall_s": time.perf_counter() - snap["t"], "input_rows": rows,
               "cached_tokens": st.cached - snap["cached"], "kv_hits": hits, "kv_misses": max(documents - hits, 0),
               "kv_removals": st.evictions - snap["evictions"], "kv_recomputations": st.replays - snap["replays"],
               "peak_gpu_bytes": int(torch.cuda.max_memory_allocated(self.device)) if self.on_gpu else 0,
               "gpu_s": (st.gpu_ms - snap["gpu_ms"]) / 1e3, "chunks": st.passes - snap["passes"],
               "reused_documents": hits, "replays": st.replays - snap["replays"]}
        out.update(extra)
        return out

    def _attention_path(self) -> str:
        """EngineConfig.attention: "tree" or "unified" as asked; None lets each chunk choose by
        the cost rule (engine/chunk.py: tree_saves)."""
        return {"tree": "tree", "unified": "unified"}.get(self.config.attention, "auto")

    def _set_answer_rows(self, ids):
        w = getattr(self.model, "w", None)
        (w if w is not None and hasattr(w, "set_answer_rows") else self.model).set_answer_rows(ids)

    # ------------------------------------------------------------ regions
    def tokenize_doc(self, doc) -> np.ndarray:
        if isinstance(doc, np.ndarray):
            return doc.astype(np.int32)
        if isinstance(doc, (bytes, bytearray, memoryview)):
            # an image document (AI.IMAGE): the vision tower reads it
            if self.images is None:
                from quail_b200.api.config import Refusal, RefusalError
                raise RefusalError(Refusal(reasons=(f"{self.cfg.name!r} has no vision tower to read an image",),
                                           constraint="unsupported_function"))
            return self.images.add(bytes(doc))
        if isinstance(doc, (list, tuple)) and (not doc or isinstance(doc[0], (int, np.integer))):
            return np.asarray(doc, dtype=np.int32)
        return self.tokenizer.encode("" if doc is None else str(doc))

    token_store = None      # engine.token_store.TokenStore shared by a session's queries

    def tokenize_docs(self, docs: list) -> list[np.ndarray]:
        """Token ids of every document; text goes through the tokenizer in one batch when it has
        one, and through the session's token store when the engine has one."""
        batch = getattr(self.tokenizer, "encode_batch", None)
        texts = [i for i, d in enumerate(docs) if d is None or isinstance(d, str)]
        out = [None] * len(docs)
        if texts and self.token_store is not None:
            enc = batch if batch is not None else (lambda xs: [self.tokenizer.encode(x) for x in xs])
            for i, ids in zip(texts, self.token_store.encode_all(["" if docs[i] is None else docs[i]
                                                                  for i in texts], enc)):
                out[i] = ids
        elif batch is not None and len(texts) > 1:
            for i, ids in zip(texts, batch(["" if docs[i] is None else docs[i] for i in texts])):
                out[i] = ids
        return [self.tokenize_doc(d) if o is None else o for d, o in zip(docs, out)]

    def run_region(self, preamble: str, docs: list, calls: list[CallSpec], *, on_rows=None,
                   stop=None) -> RegionOutput:
        """Ask `calls` over `docs`; values per input row.

        on_rows(rows, values): called as each distinct document's chain finishes, with the
        input rows that share it and their SQL values (streamed answers).
        stop(): checked between forward passes; True ends the region early, and the rows
        not finished by then come back with no values (stats["stopped"] is set).
        """
        return self._run_region(preamble, docs, calls, on_rows, stop)

    def _run_set_region(self, preamble: str, docs: list, calls: list[CallSpec], on_rows, stop) -> RegionOutput:
        """A region on a set-attention model: pass groups of questions over each document
        (engine/set_passes.py); no KV is kept between passes."""
        from quail_b200.api.config import Refusal, RefusalError
        from quail_b200.engine import set_passes as SP
        from quail_b200.sql import guards as G
        cfg, tok = self.cfg, self.tokenizer
        t0 = time.perf_counter()
        keys, uniq, where, rep = {}, [], [], []
        guarded = [c.guard for c in calls if c.guard is not None]
        for i, t in enumerate(self.tokenize_docs(docs)):
            k = t.tobytes()
            if guarded:
                k = (k, tuple(G.signature(g, i) for g in guarded))
            if k not in keys:
                keys[k] = len(uniq)
                uniq.append(t)
                rep.append(i)
            where.append(keys[k])
        yes_sp, no_sp = cfg.answer_spellings or (P.TRUE_SPELLINGS, P.FALSE_SPELLINGS)
        yes, no = tok.answer_ids(list(yes_sp)), tok.answer_ids(list(no_sp))
        end_slot = len(tok.encode("\nend:"))     # the start slot's row, counted back from the end slot
        qs = []
        for c in calls:
            body = np.asarray(tok.encode(c.tail), dtype=np.int32)
            if c.kind in ("filter", "score"):
                q = SP.SetQuestion("yes_no" if c.kind == "filter" else "score", body, c.name, yes=yes, no=no)
            elif c.kind == "classify":
                codes = c.letters or P.code_candidates(len(c.labels))
                q = SP.SetQuestion("choice", body, c.name, options=[[int(tok.encode(x)[0])] for x in codes])
            elif c.kind == "extract":
                q = SP.SetQuestion("read", body, c.name, slots=(end_slot, 0))
            else:
                raise RefusalError(Refusal(reasons=(f"{c.kind} decodes text, which the set-attention model "
                                                    f"{cfg.name!r} does not",), constraint="unsupported_function"))
            q.drops = c.drops
            if c.guard is not None:
                deps = G.calls_of(c.guard)
                q.after = tuple(j for j, o in enumerate(calls) if o.name in deps)
                q.when = (lambda r, vals, g=c.guard: G.asks(g, rep[r], self._sql_values(calls, vals, G.calls_of(g))))
            qs.append(q)
        # pass groups: a dropping filter closes its group; a call reading an answer of the
        # current group opens the next one
        groups, cur = [], []
        for j, q in enumerate(qs):
            if cur and set(q.after) & set(cur):
                groups.append(cur)
                cur = []
            cur.append(j)
            if q.kind == "yes_no" and q.drops:
                groups.append(cur)
                cur = []
        if cur:
            groups.append(cur)
        head = tok.encode(preamble)
        header = np.asarray(tok.encode(SP.D1_HEADER), dtype=np.int32)
        states = [np.concatenate([head, u, header]).astype(np.int32) for u in uniq]
        spans = [(len(head), len(u)) for u in uniq]
        region = SP.SetRegion(self.model, self._head_for_set(), self.chunk_tokens, cfg.set_size, header,
                              cfg.answer_temperature, cfg.read_span_tokens, cfg.read_found)
        values = [dict() for _ in uniq]
        kept = [True] * len(uniq)
        stopped = False
        for g in groups:
            if stop is not None and stop():
                stopped = True
                break
            # documents by the calls of this group their guards ask
            by_calls: dict = {}
            for d in range(len(uniq)):
                if not kept[d]:
                    continue
                ask = tuple(j for j in g if qs[j].when is None or qs[j].when(d, values[d]))
                if ask:
                    by_calls.setdefault(ask, []).append(d)
            for ask, who in by_calls.items():
                sub = [qs[j] for j in ask]
                got = region.ask(states, spans, sub, who)
                for d in who:
                    for k, j in enumerate(ask):
                        ans, extra = got[(d, k)]
                        c = calls[j]
                        if c.kind == "classify":
                            values[d][c.name] = ans
                            if c.probabilities:
                                values[d][c.name + "#probs"] = [float(x) for x in extra]
                        elif c.kind == "extract":
                            values[d][c.name] = (None if ans is None
                                                 else tok.decode(uniq[d][ans[0]:ans[1] + 1]).strip() or None)
                        else:
                            values[d][c.name] = ans
                            if c.kind == "filter" and c.drops and not ans:
                                kept[d] = False
        out_vals = []
        for u in where:
            v = dict(values[u])
            for c in calls:
                if c.kind == "classify" and c.name in v:
                    v[c.name] = c.labels[v[c.name]]
            out_vals.append(v)
        if on_rows is not None:
            rows_of: dict = {}
            for i, u in enumerate(where):
                rows_of.setdefault(u, []).append(i)
            for u, rows in rows_of.items():
                on_rows(rows, out_vals[rows[0]])
        st = region.stats
        stats = {"passes": st["chunks"], "fresh_tokens": st["fresh_tokens"], "documents": len(uniq),
                 "rows": len(docs), "asked": st["asked"], "set_passes": st["passes"], "chunks": st["chunks"],
                 "input_rows": len(docs), "kv_misses": len(uniq), "wall_s": time.perf_counter() - t0,
                 "output_rows": sum(1 for u in where if kept[u])}
        if stopped:
            stats["stopped"] = True
        return RegionOutput(values=out_vals, stats=stats)

    def _head_for_set(self):
        m = self.model
        return m.head

    def _run_region(self, preamble: str, docs: list, calls: list[CallSpec], on_rows, stop) -> RegionOutput:
        from quail_b200.engine.stage_executor import QueryCancelled
        if self.cfg.set_attention:
            return self._run_set_region(preamble, docs, calls, on_rows, stop)
        from quail_b200.engine.region import Call, RegionRun
        from quail_b200.sql import guards as G
        tok = self.tokenizer
        # one read per distinct document (and, with guards, per distinct guard inputs)
        guarded = [c.guard for c in calls if c.guard is not None]
        keys, uniq, where, rep = {}, [], [], []
        if self.images is not None:
            self.images.clear()
        toks = self.tokenize_docs(docs)
        if self.images is not None:
            self.images.encode(self.vision)
        for i, t in enumerate(toks):
            k = t.tobytes()
            if guarded:
                k = (k, tuple(G.signature(g, i) for g in guarded))
            if k not in keys:
                keys[k] = len(uniq)
                uniq.append(t)
                rep.append(i)
            where.append(keys[k])
        if self.cfg.role == "reranker":
            # a Qwen3 reranker answers "yes" or "no" (lowering.rs:549-551)
            true_ids, false_ids = tok.answer_ids(["yes"]), tok.answer_ids(["no"])
        else:
            true_ids = tok.answer_ids(P.TRUE_SPELLINGS)
            false_ids = tok.answer_ids(P.FALSE_SPELLINGS)
        both = set(true_ids) & set(false_ids)
        true_ids = [i for i in true_ids if i not in both]
        false_ids = [i for i in false_ids if i not in both]
        answer: list[int] = []

        def col(i: int) -> int:
            if i not in answer:
                answer.append(i)
            return answer.index(i)

        from quail_b200.api.config import Refusal, RefusalError
        for c in calls:
            if (c.kind == "features") != self.cfg.has_sae:
                why = ("AI.SAE_FEATURES needs a model with a sparse autoencoder spec" if c.kind == "features"
                       else f"{self.cfg.name} serves AI.SAE_FEATURES only")
                raise RefusalError(Refusal(reasons=(why,), constraint="unsupported_function"))
        decision = self.cfg.role == "decision"
        lettered = self.cfg.readout == "slot_lm"
        canvas = self.cfg.canvas_tokens > 0
        for c in calls:
            why = None
            if lettered and not c.letters:
                why = f"{c.kind} is not a call {self.cfg.name!r} answers: it answers with an option letter"
            elif canvas and c.kind in ("map", "extract", "features"):
                why = (f"{c.kind} needs a model that decodes token by token; {self.cfg.name!r} answers in one "
                       f"denoising step at its canvas row")
            elif canvas and c.kind == "classify" and not c.letters:
                why = f"{self.cfg.name!r} classifies under the letters rule (a letter per label)"
            elif decision and not lettered and c.segments is None:
                why = f"{c.kind} is not a call {self.cfg.name!r} answers: its head scores listed options"
            elif not decision and not canvas and (c.segments is not None or c.letters):
                why = f"an option-scoring prompt needs a decision model, not {self.cfg.name!r}"
            elif self.cfg.role == "reranker" and c.kind != "score":
                why = "a reranker model can only be used with AI.SCORE"
            if why:
                raise RefusalError(Refusal(reasons=(why,), constraint="unsupported_function"))
        rcalls = []
        for c in calls:
            offsets = ()
            if c.segments is not None:
                parts = [tok.encode(seg) for seg in c.segments]
                suffix = np.concatenate(parts).astype(np.int32) if parts else np.zeros(0, np.int32)
                lens = [len(p) for p in parts]
                # distance of each read segment's last token before the prompt's last row (lowering.rs:51-72)
                offsets = tuple(sum(lens[i + 1:]) for i in c.read) + (0,)
            else:
                suffix = tok.encode(c.tail)
            answer_canvas = canvas and c.kind == "classify" and self.cfg.canvas_answer_rows > 0
            if canvas and not answer_canvas:
                # the canvas row after the question: the answer is read there
                from quail_b200.models.gemma4 import canvas_ids
                suffix = np.concatenate([suffix, canvas_ids(self.cfg)]).astype(np.int32)
            rc = Call(kind=c.kind, suffix=suffix, name=c.name, max_tokens=c.max_tokens,
                      stop_ids=tuple(tok.eos_ids), probabilities=c.probabilities, pooling=c.pooling,
                      offsets=offsets, copy=c.kind == "extract", drops=c.drops)
            if answer_canvas:
                # a classification reads row 0 of an answer canvas after the question (draws
                # repeat an uncertain first answer)
                from quail_b200.models.gemma4 import CANVAS_ENTROPY_NATS
                from quail_b200.models.gemma4 import answer_canvas as make_canvas
                rc.canvas = (lambda r, d: make_canvas(self.cfg, r, d))
                rc.draws = max(1, int(self.config.canvas_draws))
                rc.entropy = CANVAS_ENTROPY_NATS
            if c.stop is not None and c.kind in ("map", "extract"):
                rc.stop_test = (lambda r, gen, c=c: self._stop_decision(c, gen))
            if c.guard is not None:
                deps = G.calls_of(c.guard)
                rc.after = tuple(j for j, o in enumerate(calls) if o.name in deps)
                rc.when = (lambda r, vals, g=c.guard:
                           G.asks(g, rep[r], self._sql_values(calls, vals, G.calls_of(g))))
            if c.letters:
                # the slot_lm readout: the LM head's logit of each option's letter at the last row
                ids = []
                for code in c.letters:
                    t = tok.encode(code)
                    if len(t) != 1:
                        raise RefusalError(Refusal(
                            reasons=(f"option code {code!r} is not one token of this tokenizer",),
                            constraint="unsupported_function"))
                    ids.append(int(t[0]))
                if c.kind in ("filter", "score"):
                    rc.true_cols, rc.false_cols = [col(ids[0])], [col(ids[1])]
                else:
                    rc.letter_cols = [col(i) for i in ids]
            elif offsets:
                pass
            elif c.kind in ("filter", "score"):
                rc.true_cols = [col(i) for i in true_ids]
                rc.false_cols = [col(i) for i in false_ids]
            elif c.kind == "classify":
                for label in c.labels:
                    ids = tok.encode(str(label))
                    if len(ids) == 0:
                        raise ValueError("an empty classification label")
                    rc.labels.append(ids)
                    rc.label_cols.append([col(int(i)) for i in ids])
            rcalls.append(rc)
        if not answer:
            answer = [0]
        self._set_answer_rows(answer)
        ex = self.executor
        interrupt = getattr(self, "interrupt", None)
        stopped = [False]

        def asked_stop():
            # latched: a stop hook that answers True once is not asked again
            if stop is not None and not stopped[0]:
                stopped[0] = bool(stop())
            return stopped[0]
        checks = [f for f in (interrupt.is_set if interrupt is not None else None,
                              asked_stop if stop is not None else None) if f is not None]
        ex.should_stop = (lambda: any(f() for f in checks)) if checks else None
        snap = self._snapshot()
        prefix_ids = tok.encode(preamble)
        if self.cfg.bidirectional:
            # document-isolated: the preamble and the layout's close are part of every document's block
            close = (tok.encode(P.MAMMOTH_DOCUMENT_CLOSE) if self.cfg.prompt_layout == "mammoth"
                     else np.zeros(0, np.int32))
            blocks = [np.concatenate([prefix_ids, u, close]).astype(np.int32) for u in uniq]
            run = RegionRun(ex, np.zeros(0, np.int32), blocks, rcalls, answer_width=len(answer), isolated=True)
        else:
            run = RegionRun(ex, prefix_ids, uniq, rcalls, answer_width=len(answer),
                            decision=getattr(self.model, "decision", None))
        if self.retention:
            # document KV stays in the arena for later regions with the same instruction prefix
            import hashlib
            ph = hashlib.blake2b(np.asarray(prefix_ids, np.int32).tobytes(), digest_size=8).hexdigest()
            keys = [("ret", ph, hashlib.blake2b(u.tobytes(), digest_size=12).hexdigest()) for u in uniq]
            run.retain_key = lambda r: keys[r]
            run.retained_earlier = frozenset(self._retained_keys)
            self._retained_keys.update(keys)
        rows_of: dict = {}
        for i, u in enumerate(where):
            rows_of.setdefault(u, []).append(i)

        def sql_values(u):
            v = dict(run.results[u].values)
            for c in calls:
                if c.kind in ("map", "extract") and c.name in v:
                    v[c.name] = tok.decode(v[c.name])
                if c.kind == "classify" and c.name in v:
                    v[c.name] = c.labels[v[c.name]]
            return v

        finished: set = set()

        def finish(u):
            finished.add(u)
            if on_rows is not None:
                on_rows(rows_of[u], sql_values(u))
        run.on_finish = finish
        from quail_b200.utils import progress
        kinds = ", ".join(sorted({c.kind for c in calls}))
        with progress.count(f"{kinds} over {len(uniq)} documents", len(uniq), " docs") as bar:
            run.progress = bar
            try:
                results = run.run()
            except QueryCancelled:
                if not stopped[0] or (interrupt is not None and interrupt.is_set()):
                    raise
                # stopped on request: the rows finished so far keep their answers
                values = [sql_values(u) if u in finished else {} for u in where]
                return RegionOutput(values=values, stats=self._metrics(snap, len(finished), len(docs), run.asked,
                                                                         stopped=True))
        progress.say(f"{ex.stats.passes - snap['passes']} passes, {ex.stats.tokens - snap['tokens']} fresh tokens",
                     detail=True)
        if self.on_gpu:
            from quail_b200 import ops
            err = ops.read_and_clear_error(self.device.index)
            if err:
                raise RuntimeError(f"a kernel's bounded wait ran out (code {err})")
        values = [sql_values(u) for u in where]
        del results
        stats = self._metrics(snap, len(uniq), len(docs), run.asked,
                              output_rows=sum(1 for u in where if run.results[u].kept))
        if run.stopped_early:
            stats["stopped_early"] = run.stopped_early
        return RegionOutput(values=values, stats=stats)

    def run_pairs(self, preamble: str, anchors: list, pairs: list, call: CallSpec) -> RegionOutput:
        """An AI join's region: anchor documents (each prefilled once) and (anchor index, other
        document) pairs; `call` (AI.IF or AI.SCORE) is asked once per pair. Values per pair."""
        from quail_b200.api.config import Refusal, RefusalError
        from quail_b200.engine.region import Call, PairRun
        if self.cfg.role != "generative" or self.cfg.set_attention or self.cfg.canvas_tokens:
            raise RefusalError(Refusal(reasons=(f"an AI join's pair questions need a generative model that keeps "
                                                f"KV, not {self.cfg.name!r}",), constraint="unsupported_function"))
        tok = self.tokenizer
        true_ids = tok.answer_ids(P.TRUE_SPELLINGS)
        false_ids = tok.answer_ids(P.FALSE_SPELLINGS)
        both = set(true_ids) & set(false_ids)
        answer = [i for i in true_ids if i not in both] + [i for i in false_ids if i not in both]
        nt = len([i for i in true_ids if i not in both])
        self._set_answer_rows(answer)
        rc = Call(kind=call.kind, suffix=tok.encode(call.tail), name=call.name,
                  true_cols=list(range(nt)), false_cols=list(range(nt, len(answer))))
        a_tok = self.tokenize_docs(list(anchors))
        o_tok = self.tokenize_docs([t for _, t in pairs])
        ex = self.executor
        snap = self._snapshot()
        run = PairRun(ex, tok.encode(preamble), a_tok, [(i, o) for (i, _), o in zip(pairs, o_tok)], rc,
                      answer_width=len(answer))
        from quail_b200.utils import progress
        with progress.count(f"join over {len(anchors)} anchors", len(pairs), " pairs") as bar:
            run.progress = bar
            values = run.run()
        if self.on_gpu:
            from quail_b200 import ops
            err = ops.read_and_clear_error(self.device.index)
            if err:
                raise RuntimeError(f"a kernel's bounded wait ran out (code {err})")
        stats = self._metrics(snap, sum(1 for a in a_tok if len(a)), len(pairs), run.asked, pairs=len(pairs),
                              evaluated_document_pairs=len(pairs))
        return RegionOutput(values=[{call.name: v} for v in values], stats=stats)

    def _stop_decision(self, c: CallSpec, generated) -> str:
        """"stop" once call c's WHERE test is decided on the answer's text so far."""
        from quail_b200.sql.partial import NOT_TRUE, TRUE, partial_text
        d = c.stop(partial_text(self.tokenizer.decode(generated)))
        return "stop" if d == NOT_TRUE or (d == TRUE and c.stop_when_true) else "continue"

    def _sql_values(self, calls: list[CallSpec], raw: dict, names) -> dict:
        """The SQL values of a row's answers so far (labels, decoded text), for guard tests."""
        out = {}
        for c in calls:
            if c.name in names and c.name in raw:
                v = raw[c.name]
                if c.kind == "classify":
                    v = c.labels[v]
                elif c.kind in ("map", "extract"):
                    v = self.tokenizer.decode(v)
                out[c.name] = v
        return out

    def close(self):
        self.executor = None
        self.arena = None
        self.model = None
        if self.on_gpu:
            torch.cuda.empty_cache()
