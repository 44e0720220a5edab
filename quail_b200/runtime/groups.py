"""Model copies that span several GPUs: the worker side of tp and ep sessions.

A session with `parallel="tp"` or `"ep"` starts one worker process per GPU,
as for data parallelism, but the workers of one copy (`group_gpus` of them)
see all of the copy's GPUs (CUDA_VISIBLE_DEVICES lists them; rank r uses
device r) and join one NCCL process group at boot, over which the copy's
symmetric memory is set up. Then:

- tp: every rank of a copy runs the same region on the same rows. The
  forward pass is `parallel.tp.TPQwen3` (fused AG->GEMM / GEMM->RS kernels);
  its readout rows are summed over the ranks, so every rank's scheduler
  sees the same answers and packs the same next chunk. Rank 0 reports.
- ep: each rank runs its own rows (attention is data-parallel) through the
  MoE pipeline whose expert layers exchange tokens with every peer, so the
  ranks step their schedulers in lockstep (`parallel.ep.run_lockstep`): a
  rank with nothing left runs idle passes that still serve its experts.

The weights are the same random-init checkpoint (or the same HF files) a
one-GPU engine of the model loads, split by rank, so a copy answers what a
one-GPU copy answers (up to the order of floating-point sums).
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def group_env() -> tuple[int, int, int] | None:
    """(rank, size, port) of this worker's copy, or None for a one-GPU worker."""
    size = int(os.environ.get("QB_GROUP_SIZE", "1"))
    if size <= 1:
        return None
    return int(os.environ["QB_GROUP_RANK"]), size, int(os.environ["QB_GROUP_PORT"])


def build_group_engine(config, rank: int, size: int, port: int, timeout_s: float = 120.0):
    """Join the copy's process group and build this rank's engine of a tp / ep copy."""
    from dataclasses import replace

    from quail_b200.api.config import check_config
    from quail_b200.api.engine import ModelEngine
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.build import random_checkpoint_on

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size,
                            device_id=dev, timeout=timedelta(seconds=timeout_s))
    cpu_group = dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))
    cfg = check_config(config)
    one = replace(config, gpus=1, parallel="dp", group_gpus=None)
    from quail_b200.planner.budgets import Budgets
    chunk = config.chunk_tokens or Budgets.for_model(cfg, config.device, gpus=1).chunk_tokens
    if config.weights:
        from quail_b200.models.weights import load_checkpoint
        ckpt = load_checkpoint(config.weights, device=dev)
    else:
        ckpt = random_checkpoint_on(cfg, dev, seed=config.seed)
    free = torch.cuda.mem_get_info(dev)[0]
    if config.parallel == "tp":
        from quail_b200.parallel.tp import TPQwen3
        model = TPQwen3(cfg, dist.group.WORLD, seed=config.seed, max_tokens=chunk + 4096, full_weights=ckpt)
        del ckpt
        torch.cuda.empty_cache()
        kv_heads = cfg.num_kv_heads // size
        page_tokens = 128
        pages = _pages(cfg, kv_heads, page_tokens, dev, share=0.8)
        arena = KVArena(cfg.layers, pages, page_tokens, kv_heads, cfg.head_dim, device=dev)
        engine = ModelEngine.from_replica(one, model, arena)
        engine.group = (rank, size)
        return engine
    from quail_b200.models.qwen3_moe import Qwen3MoePipeline, Qwen3MoeWeights
    E = cfg.num_experts
    lo, hi = rank * E // size, (rank + 1) * E // size
    weights = Qwen3MoeWeights(cfg, ckpt, dev, experts=range(lo, hi), head_rows=range(8), seed=config.seed)
    del ckpt
    pipe = Qwen3MoePipeline(cfg, weights, max_tokens=chunk + 256, group=dist.group.WORLD)
    torch.cuda.empty_cache()
    page_tokens = int(config.extra.get("page_tokens", 16))
    pages = _pages(cfg, cfg.num_kv_heads, page_tokens, dev, share=0.7)
    arena = KVArena(cfg.layers, pages, page_tokens, cfg.num_kv_heads, cfg.head_dim, device=dev)
    engine = ModelEngine.from_replica(one, pipe, arena)
    engine.executor = LockstepExecutor(pipe, arena, engine.chunk_tokens, cpu_group)
    engine.group = (rank, size)
    del free
    return engine


def _pages(cfg, kv_heads: int, page_tokens: int, dev, share: float) -> int:
    """Arena pages from the free memory left after the weights (`share` of it)."""
    free, _ = torch.cuda.mem_get_info(dev)
    per_page = cfg.layers * 2 * page_tokens * kv_heads * cfg.head_dim * 2
    return max(64, int(free * share) // per_page)


class LockstepExecutor:
    """A stage executor whose run() steps in lockstep with the other ranks of an ep copy."""

    def __new__(cls, pipe, arena, chunk_tokens: int, cpu_group):
        from quail_b200.engine.stage_executor import StageExecutor

        class _Lockstep(StageExecutor):
            def run(self):
                from quail_b200.parallel.ep import run_lockstep
                run_lockstep(self, pipe, cpu_group)
                return self.stats

        return _Lockstep(pipe, arena, chunk_tokens)
