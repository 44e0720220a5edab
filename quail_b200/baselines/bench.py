"""The flagship AI.IF workload through stock vLLM, one request per row (a same-box comparison).

    python -m quail_b200.baselines.bench [--rows 20000] [--model qwen3-4b-fp8]

The rows are bench.py's synthetic rows (token-id bodies lognormal(median 180,
sigma 0.6) clipped to [16, 2048], the 48-token shared template prefix, the
40-token question) on the same random-init weights, exported as a Hugging Face
checkpoint (not timed). vLLM boots (reported, not timed), answers a warm-up
batch, then every row's request in one `generate` call with prefix caching on;
the timed region is that call's wall time (the client's view: scheduling,
batching and the forward passes), so prompt tokens / s compares with the
end-to-end number of this engine's own bench line. Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import tempfile
import time


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-4b-fp8")
    ap.add_argument("--rows", type=int, default=20000)
    ap.add_argument("--warmup-rows", type=int, default=512)
    ap.add_argument("--checkpoint", default=None, help="an exported checkpoint directory to reuse")
    args = ap.parse_args(argv)
    import numpy as np
    import torch

    from quail_b200.api.config import EngineConfig
    from quail_b200.baselines.hf_export import export_checkpoint
    from quail_b200.baselines.vllm_backend import VLLMEngine, margin_of, request_tokens
    from quail_b200.models.build import SYNTHETIC_FALSE_IDS, SYNTHETIC_TRUE_IDS
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.utils.clocks import ClockSampler
    from quail_b200.utils.synthetic import make_workload

    cfg = MODEL_CONFIGS[args.model]
    t0 = time.perf_counter()
    path = args.checkpoint or export_checkpoint(cfg, tempfile.mkdtemp(prefix="qb_vllm_"), seed=0, device="cuda")
    export_s = time.perf_counter() - t0
    torch.cuda.empty_cache()
    eng = VLLMEngine(EngineConfig(model=args.model, device="b200"), checkpoint_dir=path)
    eng.llm()
    warm = make_workload(args.warmup_rows, seed=4000)
    eng._generate([request_tokens(warm.prefix, b, warm.suffix) for b in warm.bodies], 1)
    wl = make_workload(args.rows, seed=2000)
    prompts = [request_tokens(wl.prefix, b, wl.suffix) for b in wl.bodies]
    tokens = sum(len(p) for p in prompts)
    sampler = ClockSampler(0).start()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    outs = eng._generate(prompts, 1)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t1
    clocks = sampler.stop()
    kept = 0
    for o in outs:
        lp = {k: v.logprob for k, v in (o.outputs[0].logprobs[0] if o.outputs[0].logprobs else {}).items()}
        kept += margin_of(lp, SYNTHETIC_TRUE_IDS, SYNTHETIC_FALSE_IDS) > 0
    import vllm
    print(json.dumps({
        "metric": "AI.IF prompt tok/s through stock vLLM, one request per row (same box, same weights)",
        "value": round(tokens / wall, 1), "unit": "prompt tokens/s", "rows_per_second": round(args.rows / wall, 1),
        "rows": args.rows, "prompt_tokens": tokens, "wall_s": round(wall, 3), "boot_s": round(eng.boot_s, 1),
        "export_s": round(export_s, 1), "kept_rows": int(kept), "model": args.model,
        "vllm": vllm.__version__, "prefix_caching": True, "clocks": clocks,
        "mean_prompt_tokens": round(float(np.mean([len(p) for p in prompts])), 1),
        "pid": os.getpid()}), flush=True)


if __name__ == "__main__":
    main()
