"""Device-timed microbenchmarks of the hot kernels at the model shapes.

    python -m quail_b200.utils.kernel_bench [--model qwen3-4b-fp8] [--tokens 16384]

Each case is timed with CUDA events on the launching stream after warm-up,
with an L2 flush (a 512 MiB write) before every timed launch, and reported
as achieved TFLOP/s or GB/s next to the library bars the reference would
call on the same GPU (cuBLAS bf16 matmul, cuBLASLt fp8 `_scaled_mm`).
"""

from __future__ import annotations

import argparse
import json

import torch

from quail_b200 import ops
from quail_b200.models.config import MODEL_CONFIGS


def _timeit(fn, iters=10, warmup=3, flush=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def gemm_cases(cfg, T):
    H = cfg.hidden
    return [("qkv", T, cfg.qkv_dim, H), ("o_proj", T, H, cfg.q_dim), ("gate_up", T, 2 * cfg.intermediate, H),
            ("down", T, H, cfg.intermediate)]


def run(model: str, T: int, iters: int = 10) -> list[dict]:
    cfg = MODEL_CONFIGS[model]
    dev = "cuda"
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    out = []
    for name, M, N, K in gemm_cases(cfg, T):
        flops = 2.0 * M * N * K
        a = torch.randn(M, K, device=dev)
        b = torch.randn(N, K, device=dev) * 0.02
        row = {"case": name, "M": M, "N": N, "K": K}
        if cfg.fp8:
            a8, sa = ops.quantize_act(a)
            b8, sb = ops.quantize_weight(b)
            epi = ops.EPI_BF16
            if name == "gate_up":
                b8, sb = ops.interleave_gate_up(b8, sb)
                ms = _timeit(lambda: ops.gemm(a8, b8, sa=sa, sb=sb, sb_gran=64, epi=ops.EPI_SWIGLU_FP8),
                             iters, flush=flush)
            else:
                dout = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                ms = _timeit(lambda: ops.gemm(a8, b8, sa=sa, sb=sb, epi=epi, out=dout), iters, flush=flush)
            row["ours_ms"] = ms
            row["ours_tflops"] = flops / ms / 1e9
            # MX (UE8M0) block-scaled path
            a8m, sfa = ops.quantize_act_mx(a)
            if name == "gate_up":
                b8m, sfb = ops.interleave_gate_up_mx(b)
                ms_mx = _timeit(lambda: ops.gemm_mx(a8m, sfa, b8m, sfb, epi=ops.EPI_SWIGLU_FP8), iters, flush=flush)
            else:
                b8m, sfb = ops.quantize_weight_mx(b)
                dmx = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                ms_mx = _timeit(lambda: ops.gemm_mx(a8m, sfa, b8m, sfb, out=dmx), iters, flush=flush)
            row["mx_ms"] = ms_mx
            row["mx_tflops"] = flops / ms_mx / 1e9
            try:
                one = torch.ones((), device=dev)
                bt = b8.t()
                ms_l = _timeit(lambda: torch._scaled_mm(a8, bt, scale_a=one, scale_b=one, out_dtype=torch.bfloat16),
                               iters, flush=flush)
                row["cublaslt_fp8_tensorwise_ms"] = ms_l
                row["cublaslt_fp8_tensorwise_tflops"] = flops / ms_l / 1e9
            except Exception as exc:  # noqa: BLE001
                row["cublaslt_fp8_error"] = str(exc)[:120]
        ab, bb = a.bfloat16(), b.bfloat16()
        ms_c = _timeit(lambda: ab @ bb.t(), iters, flush=flush)
        row["cublas_bf16_ms"] = ms_c
        row["cublas_bf16_tflops"] = flops / ms_c / 1e9
        if not cfg.fp8:
            ms = _timeit(lambda: ops.gemm(ab, bb), iters, flush=flush)
            row["ours_ms"] = ms
            row["ours_tflops"] = flops / ms / 1e9
        out.append(row)
        del a, b
    assert ops.read_and_clear_error(0) == 0
    return out


def attention_case(cfg, tokens: int, seed: int = 0):
    """A packed chunk like the AI.IF benchmark's: 48-token shared prefix, lognormal rows."""
    import numpy as np

    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.chunk import ChunkPacker, SeqSpec
    from quail_b200.utils.synthetic import make_workload, rows_for_tokens
    wl = make_workload(rows_for_tokens(tokens), seed=seed)
    arena = KVArena(1, 4096, 128, cfg.num_kv_heads, cfg.head_dim, device="cuda")
    pool = arena.pool
    pool.alloc("p", 48)
    specs, n = [], 0
    for i, b in enumerate(wl.bodies):
        toks = np.concatenate([b, wl.suffix])
        if n + len(toks) > tokens:
            break
        pool.alloc(i, len(toks))
        specs.append(SeqSpec(reads=[("p", 48)], own_key=i, own_start=0, tokens=toks, pos_start=48, readout=True))
        n += len(toks)
    chunk = ChunkPacker(pool, "cuda").pack(specs)
    kc, vc = arena.layer(0)
    kc.normal_()
    vc.normal_()
    q = torch.randn(chunk.num_tokens, cfg.num_q_heads, 128, device="cuda").bfloat16()
    # causal FLOPs actually needed: each token attends to the prefix and its own earlier tokens
    ctx = 0.0
    for s_ in specs:
        L = len(s_.tokens)
        ctx += L * 48 + L * (L + 1) / 2
    flops = 4.0 * ctx * cfg.num_q_heads * 128
    return chunk, q, kc, vc, flops


def run_attention(model: str, tokens: int, iters: int = 10) -> dict:
    from quail_b200.ops import reference as ref
    cfg = MODEL_CONFIGS[model]
    chunk, q, kc, vc, flops = attention_case(cfg, tokens)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    ms = _timeit(lambda: ops.prefill_attention(q, kc, vc, chunk.seqs, chunk.tiles, chunk.page_list,
                                               ref.softmax_scale(128), fp8_out=True, mx=True), iters, flush=flush)
    ms_tc = _timeit(lambda: ops.prefill_attention_tc(q, kc, vc, chunk.seqs, chunk.tiles, chunk.page_list,
                                                     ref.softmax_scale(128)), iters, flush=flush)
    ms_p = _timeit(lambda: ops.prefill_attention_tc2(q, kc, vc, chunk.seqs, chunk.blocks, chunk.page_list,
                                                     ref.softmax_scale(128)), iters, flush=flush)
    assert ops.read_and_clear_error(0) == 0
    row = {"case": "prefill_attention", "tokens": chunk.num_tokens, "mma_sync_ms": ms,
           "mma_sync_useful_tflops": flops / ms / 1e9, "tcgen05_ms": ms_tc,
           "tcgen05_useful_tflops": flops / ms_tc / 1e9, "persistent_ms": ms_p,
           "persistent_useful_tflops": flops / ms_p / 1e9}
    row.update(_fa4_bar(cfg, chunk, q, kc, vc, flops, iters, flush))
    return row


def _fa4_bar(cfg, chunk, q, kc, vc, flops, iters, flush) -> dict:
    """The library bar on the same shapes: FA4 (CuTe DSL, sm100) as the reference calls it on B200.

    Each packed row is one varlen sequence whose keys are the 48 shared prefix
    tokens followed by its own tokens, contiguous (the prefix copied in front
    of every row); queries are the row's own tokens, causal with the
    bottom-right alignment, so the work equals the paged kernel's.
    """
    try:
        from vllm.vllm_flash_attn import flash_attn_varlen_func
    except Exception as exc:  # noqa: BLE001
        return {"fa4_error": f"import: {str(exc)[:160]}"}
    seqs = chunk.seqs.cpu().tolist()
    P = kc.shape[1]
    pl = chunk.page_list.cpu()
    kk, vv, cuq, cuk = [], [], [0], [0]
    for sd in seqs:
        q_len, nseg = sd[1], sd[2]
        ks, vs = [], []
        for i in range(nseg):
            ln, off = sd[4 + i], sd[8 + i]
            pages = pl[off: off + (ln + P - 1) // P].to(kc.device)
            ks.append(kc[pages].reshape(-1, kc.shape[2], kc.shape[3])[:ln])
            vs.append(vc[pages].reshape(-1, vc.shape[2], vc.shape[3])[:ln])
        k1, v1 = torch.cat(ks), torch.cat(vs)
        kk.append(k1)
        vv.append(v1)
        cuq.append(cuq[-1] + q_len)
        cuk.append(cuk[-1] + k1.shape[0])
    k_all, v_all = torch.cat(kk).contiguous(), torch.cat(vv).contiguous()
    cu_q = torch.tensor(cuq, dtype=torch.int32, device=q.device)
    cu_k = torch.tensor(cuk, dtype=torch.int32, device=q.device)
    max_q = max(b - a for a, b in zip(cuq, cuq[1:]))
    max_k = max(b - a for a, b in zip(cuk, cuk[1:]))
    qq = q[: cuq[-1]].contiguous()
    from quail_b200.ops import reference as ref
    try:
        fn = lambda: flash_attn_varlen_func(qq, k_all, v_all, max_q, cu_q, max_k, cu_seqlens_k=cu_k,  # noqa: E731
                                            softmax_scale=ref.softmax_scale(128), causal=True, fa_version=4)
        ms = _timeit(fn, iters, flush=flush)
    except Exception as exc:  # noqa: BLE001
        return {"fa4_error": f"call: {str(exc)[:200]}"}
    return {"fa4_ms": ms, "fa4_useful_tflops": flops / ms / 1e9}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-4b-fp8")
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--only", default="all", choices=["all", "gemm", "attention", "persistent"])
    args = ap.parse_args()
    if args.only in ("all", "gemm"):
        for row in run(args.model, args.tokens, args.iters):
            print(json.dumps(row))
    if args.only in ("all", "attention"):
        print(json.dumps(run_attention(args.model, args.tokens, args.iters)))
    if args.only == "persistent":
        # one case for a profiler: the persistent attention kernel alone, `iters` launches
        from quail_b200.ops import reference as ref
        cfg = MODEL_CONFIGS[args.model]
        chunk, q, kc, vc, _ = attention_case(cfg, args.tokens)
        for _ in range(args.iters):
            ops.prefill_attention_tc2(q, kc, vc, chunk.seqs, chunk.blocks, chunk.page_list, ref.softmax_scale(128))
        torch.cuda.synchronize()
        assert ops.read_and_clear_error(0) == 0


if __name__ == "__main__":
    main()
