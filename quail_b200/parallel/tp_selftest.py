"""Self-test of the fused tensor-parallel path against the one-GPU pipeline.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m quail_b200.parallel.tp_selftest

Every rank builds the same random checkpoint; the TP model runs packed
chunks (a shared prefix read by every row, rows split into prefill pieces)
through the stage executor; rank 0 then runs the same tasks through the
single-GPU MX pipeline with the unsharded weights and through the fp32 model
of the same weights. Both fp8 paths round differently (the TP path reduces
bf16 partial sums across ranks), so each is judged against the fp32 model:
the TP logits must be about as close to it as the one-GPU pipeline's. Prints
one JSON line on rank 0.
"""

from __future__ import annotations

import json
import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist


def _run(model, arena, prefix, docs, suffix, chunk_tokens):
    from quail_b200.engine.stage_executor import StageExecutor, Task
    ex = StageExecutor(model, arena, chunk_tokens, min_piece=16)
    got = {}
    ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
    for i, d in enumerate(docs):
        ex.submit(Task(key=i, tokens=np.concatenate([d, suffix]), pos_start=len(prefix), reads=[("p", len(prefix))],
                       readout=True, on_done=lambda t, row, i=i: got.__setitem__(i, row.float().cpu())))
    ex.run()
    return torch.stack([got[i] for i in range(len(docs))])


def main():
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    from quail_b200 import ops
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.config import DecoderConfig
    from quail_b200.models.qwen3 import Qwen3Pipeline, Qwen3Weights
    from quail_b200.models.weights import random_checkpoint
    from quail_b200.parallel.tp import TPQwen3

    cfg = DecoderConfig(name="tp-test", layers=2, hidden=1024, num_q_heads=16, num_kv_heads=4, head_dim=128,
                        intermediate=1024 * world // 2 if world > 2 else 1024, vocab=4096, max_position=8192)
    if cfg.intermediate % (world * 128):
        cfg = cfg.with_(intermediate=world * 256)
    ckpt = random_checkpoint(cfg, seed=11, device=dev)
    ids = list(range(16))
    tpm = TPQwen3(cfg, dist.group.WORLD, max_tokens=4096, answer_ids=ids, full_weights=ckpt)
    rng = np.random.default_rng(0)
    prefix = rng.integers(0, 4096, 48).astype(np.int32)
    docs = [rng.integers(0, 4096, n).astype(np.int32) for n in (10, 300, 64, 700, 129, 33)]
    suffix = rng.integers(0, 4096, 24).astype(np.int32)
    arena = KVArena(cfg.layers, 128, 128, cfg.num_kv_heads // world, 128, device=dev)
    got = _run(tpm, arena, prefix, docs, suffix, 1024)
    err_tp = tpm.check_errors()
    dist.barrier()
    out = {"world": world, "kernel_error": err_tp}
    if rank == 0:
        from quail_b200.models.qwen3 import Qwen3Reference
        pipe = Qwen3Pipeline(cfg, Qwen3Weights(cfg, ckpt, dev, head_rows=ids))
        arena1 = KVArena(cfg.layers, 128, 128, cfg.num_kv_heads, 128, device=dev)
        one = _run(pipe, arena1, prefix, docs, suffix, 1024)
        exact = Qwen3Reference(cfg, ckpt, device=dev, head_rows=ids)
        arena32 = KVArena(cfg.layers, 128, 128, cfg.num_kv_heads, 128, device=dev, dtype=torch.float32)
        want = _run(exact, arena32, prefix, docs, suffix, 1024)

        def rel(a, b):
            return float(((a - b).norm() / b.norm()).item())

        def agree(a, b):
            return float((a.argmax(1) == b.argmax(1)).float().mean().item())
        out.update(rel_err=rel(got, one), rel_err_tp_fp32=rel(got, want), rel_err_one_fp32=rel(one, want),
                   argmax_agree_tp_fp32=agree(got, want), argmax_agree_one_fp32=agree(one, want))
        out["ok"] = (out["rel_err_tp_fp32"] < 1.5 * out["rel_err_one_fp32"] + 0.03
                     and out["argmax_agree_tp_fp32"] >= out["argmax_agree_one_fp32"] - 0.2 and err_tp == 0)
        print(json.dumps(out), flush=True)
    dist.barrier()
    del tpm
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
