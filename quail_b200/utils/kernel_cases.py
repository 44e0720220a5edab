"""Single-kernel cases for profilers and timers: the NVFP4 GEMM and the chunked GDN layer.

    python -m quail_b200.utils.kernel_cases nvfp4 [--m 8192 --n 17408 --k 5120] [--iters 3]
    python -m quail_b200.utils.kernel_cases gdn [--mode 1] [--iters 10]

nvfp4: one qwen3.8-27b MLP-shaped NVFP4 GEMM (E2M1 operands with UE4M3
16-value block scales, per-tensor alpha), launched `iters` times after two
warm-up calls; prints the median device time and TFLOP/s.

gdn: one Gated DeltaNet layer of a packed 16k-token prefill pass in the
qwen3.5-27b geometry (16 key / 32 value heads of 128, conv width 4) over
lognormal(median 180, sigma 0.6) rows + 88 template/question tokens;
`--mode` picks the path (0 chunked on the tensor cores, 1 the per-token
recurrence, 3 chunked with the prep kernel split); prints device ms per
layer. Both are the commands the NVFP4 / GDN profiles were taken with.
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch


def _time(fn, iters: int) -> float:
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def nvfp4_case(m: int, n: int, k: int, iters: int) -> dict:
    from quail_b200 import ops
    from quail_b200.ops.quant import quantize_nvfp4
    a = torch.randn(m, k, device="cuda")
    b = torch.randn(n, k, device="cuda") * 0.05
    pa, sa, ga = quantize_nvfp4(a)
    pb, sb, gb = quantize_nvfp4(b)
    del a, b
    ms = _time(lambda: ops.gemm_nvfp4(pa, sa, pb, sb, ga * gb), iters)
    assert ops.read_and_clear_error(0) == 0
    return {"case": "gemm_nvfp4", "M": m, "N": n, "K": k, "ms": ms, "tflops": 2.0 * m * n * k / ms / 1e9}


def nvfp4_library_bar(m: int, n: int, k: int, iters: int) -> dict:
    """The same shape on FlashInfer's mm_fp4 (the reference's NVFP4 GEMM on B200), CUTLASS and
    CuTe-DSL backends, inputs quantized by FlashInfer's own nvfp4_quantize (128x4 scale layout)."""
    out = {}
    try:
        from flashinfer import SfLayout, mm_fp4, nvfp4_quantize
    except Exception as exc:  # noqa: BLE001 - the bar is recorded as unavailable
        return {"flashinfer_error": f"import: {str(exc)[:160]}"}
    a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    b = (torch.randn(n, k, device="cuda") * 0.05).bfloat16()
    ga = (448 * 6) / a.float().abs().max()
    gb = (448 * 6) / b.float().abs().max()
    a4, asf = nvfp4_quantize(a, ga, sfLayout=SfLayout.layout_128x4, do_shuffle=False)
    b4, bsf = nvfp4_quantize(b, gb, sfLayout=SfLayout.layout_128x4, do_shuffle=False)
    alpha = (1.0 / (ga * gb)).float().reshape(1)
    for backend in ("cutlass", "cute-dsl"):
        try:
            ms = _time(lambda: mm_fp4(a4, b4.T, asf, bsf.T, alpha, torch.bfloat16, None, backend=backend), iters)
            out[f"flashinfer_{backend}_ms"] = ms
            out[f"flashinfer_{backend}_tflops"] = 2.0 * m * n * k / ms / 1e9
        except Exception as exc:  # noqa: BLE001
            out[f"flashinfer_{backend}_error"] = str(exc)[:200]
    return out


def gdn_library_bar(iters: int, tokens: int = 16384) -> dict:
    """FlashInfer's chunked gated delta rule prefill (the reference's GDN path on B200) on the
    same sequences and head geometry, if it imports and runs here."""
    try:
        from flashinfer.gdn_prefill import chunk_gated_delta_rule
    except Exception as exc:  # noqa: BLE001
        return {"flashinfer_gdn_error": f"import: {str(exc)[:160]}"}
    rng = np.random.default_rng(0)
    lens = np.clip(rng.lognormal(np.log(180), 0.6, 400), 16, 2048).astype(int) + 88
    lens = lens[np.cumsum(lens) <= tokens]
    T = int(lens.sum())
    Hk, Hv, d = 16, 32, 128
    dev = "cuda"
    q = torch.randn(T, Hk, d, device=dev, dtype=torch.bfloat16)
    kk = torch.nn.functional.normalize(torch.randn(T, Hk, d, device=dev), dim=-1).bfloat16()
    v = torch.randn(T, Hv, d, device=dev, dtype=torch.bfloat16)
    g = -torch.rand(T, Hv, device=dev) * 0.1
    beta = torch.rand(T, Hv, device=dev)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int64, device=dev)
    try:
        ms = _time(lambda: chunk_gated_delta_rule(q, kk, v, g, beta, cu_seqlens=cu), iters)
    except Exception as exc:  # noqa: BLE001
        return {"flashinfer_gdn_error": f"call: {str(exc)[:200]}"}
    return {"flashinfer_gdn_ms": ms}


def gdn_case(mode: int, iters: int, tokens: int = 16384) -> dict:
    from quail_b200 import ops
    dev = "cuda"
    torch.manual_seed(0)
    Hk, Hv, dk, dv, W = 16, 32, 128, 128, 4
    C = 2 * Hk * dk + Hv * dv
    rng = np.random.default_rng(0)
    lens = np.clip(rng.lognormal(np.log(180), 0.6, 400), 16, 2048).astype(int) + 88
    lens = lens[np.cumsum(lens) <= tokens]
    T, S = int(lens.sum()), len(lens)
    proj = (torch.randn(T, C + Hv * dv + 2 * Hv, device=dev) * 0.5).bfloat16()
    conv_w = torch.randn(C, W, device=dev) * 0.3
    A_log = torch.log(1 + 15 * torch.rand(Hv, device=dev))
    dt_bias = torch.randn(Hv, device=dev) - 3
    norm_w = torch.ones(dv, device=dev).bfloat16()
    seqs = torch.zeros(S, 12, dtype=torch.int32)
    q0 = 0
    for i, n in enumerate(lens):
        seqs[i, 0], seqs[i, 1], seqs[i, 2], seqs[i, 4] = q0, int(n), 1, int(n)
        q0 += int(n)
    sio = torch.tensor([[-1, i] for i in range(S)], dtype=torch.int32)
    conv_state = torch.zeros(S, 1, W - 1, C, device=dev)
    ssm = torch.zeros(S, 1, Hv, dk, dv, device=dev)
    conv_out = torch.empty(T, C, device=dev)
    o = torch.empty(T, Hv * dv, device=dev)
    y = torch.empty(T, Hv * dv, dtype=torch.bfloat16, device=dev)
    sq, sd = seqs.to(dev), sio.to(dev)

    def layer():
        ops.native().gdn_layer(proj, conv_w, A_log, dt_bias, norm_w, sq, sd, conv_state, ssm, 0, Hk, Hv, dk, dv,
                               1e-6, conv_out, o, y, mode)
    ms = _time(layer, iters)
    assert ops.read_and_clear_error(0) == 0
    return {"case": "gdn_layer", "mode": mode, "tokens": T, "sequences": S, "ms": ms}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["nvfp4", "gdn"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=17408)
    ap.add_argument("--k", type=int, default=5120)
    ap.add_argument("--mode", type=int, default=0)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--bar", action="store_true", help="also time the library kernel the reference calls")
    args = ap.parse_args()
    if args.case == "nvfp4":
        row = nvfp4_case(args.m, args.n, args.k, args.iters)
        if args.bar:
            row.update(nvfp4_library_bar(args.m, args.n, args.k, args.iters))
    else:
        row = gdn_case(args.mode, args.iters)
        if args.bar:
            row.update(gdn_library_bar(args.iters))
    print(json.dumps(row))


if __name__ == "__main__":
    main()
