"""Self-test of the expert-parallel MoE path against the one-GPU pipeline.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m quail_b200.parallel.ep_selftest

Every rank builds the same replicated weights and its own E / W experts
(per-layer and per-expert random streams), runs its own documents (same
lengths on every rank, different tokens, so every rank runs the same number
of chunks and MoE layers) through the stage executor with expert
parallelism, then runs the same documents through a one-rank pipeline that
holds all experts and compares the readout logits; then the same with the
NCCL all-to-all baseline path. The expert math of a row
does not depend on where it runs, so the two agree to rounding. Prints one
JSON line on rank 0 (max error over ranks).
"""

from __future__ import annotations

import json
import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist


def main():
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.config import QWEN3_MOE_GPU_TINY
    from quail_b200.models.qwen3_moe import Qwen3MoePipeline, Qwen3MoeWeights
    from quail_b200.parallel.tp_selftest import _run

    cfg = QWEN3_MOE_GPU_TINY.with_(vocab=4096, max_position=8192)
    E = cfg.num_experts
    ids = list(range(16))
    lo, hi = rank * E // world, (rank + 1) * E // world
    ep = Qwen3MoePipeline(cfg, Qwen3MoeWeights(cfg, None, dev, experts=range(lo, hi), head_rows=ids, seed=4),
                          max_tokens=1024, group=dist.group.WORLD)
    rng = np.random.default_rng(100 + rank)
    lens = (10, 300, 64, 700, 129, 33)
    prefix = np.random.default_rng(0).integers(0, 4096, 48).astype(np.int32)
    docs = [rng.integers(0, 4096, n).astype(np.int32) for n in lens]
    suffix = np.random.default_rng(1).integers(0, 4096, 24).astype(np.int32)
    arena = KVArena(cfg.layers, 128, 128, cfg.num_kv_heads, 128, device=dev)
    got = _run(ep, arena, prefix, docs, suffix, 1024)
    err_ep = ops.read_and_clear_error(local)
    dist.barrier()
    # the NCCL all-to-all baseline on the same weights and rows
    ep.ep.comm = "nccl"
    arena_n = KVArena(cfg.layers, 128, 128, cfg.num_kv_heads, 128, device=dev)
    got_n = _run(ep, arena_n, prefix, docs, suffix, 1024)
    err_ep = max(err_ep, ops.read_and_clear_error(local))
    dist.barrier()
    one = Qwen3MoePipeline(cfg, Qwen3MoeWeights(cfg, None, dev, head_rows=ids, seed=4), max_tokens=1024)
    arena1 = KVArena(cfg.layers, 128, 128, cfg.num_kv_heads, 128, device=dev)
    want = _run(one, arena1, prefix, docs, suffix, 1024)
    err_one = ops.read_and_clear_error(local)
    rel = torch.tensor([float(((got - want).norm() / want.norm()).item()), float(err_ep), float(err_one),
                        float(((got_n - want).norm() / want.norm()).item())], device=dev)
    dist.all_reduce(rel, op=dist.ReduceOp.MAX)
    out = {"world": world, "rel_err": rel[0].item(), "rel_err_nccl": rel[3].item(),
           "kernel_error": int(rel[1].item()), "one_rank_error": int(rel[2].item())}
    out["ok"] = (out["rel_err"] < 1e-2 and out["rel_err_nccl"] < 1e-2 and out["kernel_error"] == 0
                 and out["one_rank_error"] == 0)
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    del ep
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
