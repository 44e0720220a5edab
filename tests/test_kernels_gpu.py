"""Kernel numerics against the plain-PyTorch fp32 statement of each op."""

import pytest
import torch

from quail_b200 import ops
from quail_b200.ops import reference as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp(min=1e-12)).item()


@pytest.fixture(autouse=True)
def _no_kernel_errors():
    torch.manual_seed(0)
    yield
    assert ops.read_and_clear_error(0) == 0


@pytest.mark.parametrize("M,N,K,bn", [(128, 256, 128, 256), (300, 512, 1024, 256), (1000, 384, 640, 128),
                                       (77, 2560, 2560, 256)])
def test_gemm_bf16(M, N, K, bn):
    a = torch.randn(M, K, device=DEV).bfloat16()
    b = torch.randn(N, K, device=DEV).bfloat16()
    d = ops.gemm(a, b, bn=bn)
    want = a.float() @ b.float().t()
    assert rel_err(d, want) < 1e-2


@pytest.mark.parametrize("M,N,K,bn", [(128, 256, 128, 256), (300, 512, 1024, 256), (1000, 384, 640, 128),
                                       (2048, 6144, 2560, 256), (33, 2560, 9728, 256)])
def test_gemm_fp8_blockscaled(M, N, K, bn):
    a = torch.randn(M, K, device=DEV)
    b = torch.randn(N, K, device=DEV) * 0.02
    a8, sa = ops.quantize_act(a)
    b8, sb = ops.quantize_weight(b)
    d = ops.gemm(a8, b8, sa=sa, sb=sb, bn=bn)
    want = ops.dequantize_act(a8, sa) @ ops.dequantize_weight(b8, sb).t()
    assert rel_err(d, want) < 5e-3


def test_gemm_fp8_residual_epilogue():
    M, N, K = 500, 2560, 1024
    a8, sa = ops.quantize_act(torch.randn(M, K, device=DEV))
    b8, sb = ops.quantize_weight(torch.randn(N, K, device=DEV) * 0.02)
    res = torch.randn(M, N, device=DEV).bfloat16()
    want = ops.dequantize_act(a8, sa) @ ops.dequantize_weight(b8, sb).t() + res.float()
    ops.gemm(a8, b8, sa=sa, sb=sb, epi=ops.EPI_RESIDUAL, out=res, residual=res)
    assert rel_err(res, want) < 5e-3


def test_gemm_bf16_residual_epilogue():
    M, N, K = 260, 512, 512
    a = torch.randn(M, K, device=DEV).bfloat16()
    b = torch.randn(N, K, device=DEV).bfloat16()
    res = torch.randn(M, N, device=DEV).bfloat16()
    want = a.float() @ b.float().t() + res.float()
    ops.gemm(a, b, epi=ops.EPI_RESIDUAL, out=res, residual=res)
    assert rel_err(res, want) < 1e-2


def test_gemm_fp8_swiglu_epilogue():
    M, inter, K = 700, 1024, 1024
    x = torch.randn(M, K, device=DEV)
    w = torch.randn(2 * inter, K, device=DEV) * 0.05
    a8, sa = ops.quantize_act(x)
    w8, sw = ops.quantize_weight(w)
    wi, swi = ops.interleave_gate_up(w8, sw)
    y8, ys = ops.gemm(a8, wi, sa=sa, sb=swi, sb_gran=64, epi=ops.EPI_SWIGLU_FP8)
    gu = ops.dequantize_act(a8, sa) @ ops.dequantize_weight(w8, sw).t()
    want = ref.silu_mul(gu[:, :inter], gu[:, inter:])
    got = ops.dequantize_act(y8, ys)
    assert rel_err(got, want) < 4e-2


def test_gemm_bf16_swiglu_epilogue():
    M, inter, K = 300, 512, 512
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(2 * inter, K, device=DEV) * 0.05).bfloat16()
    wi = ops.interleave_gate_up(w)
    y = ops.gemm(x, wi, epi=ops.EPI_SWIGLU_BF16)
    gu = x.float() @ w.float().t()
    want = ref.silu_mul(gu[:, :inter], gu[:, inter:])
    assert rel_err(y, want) < 1e-2


@pytest.mark.parametrize("H", [1024, 2560, 4096])
def test_rmsnorm_quant(H):
    T = 333
    x = torch.randn(T, H, device=DEV).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=DEV)).bfloat16()
    y8, ys = ops.rmsnorm_quant(x, w, 1e-6)
    want = ref.rmsnorm(x, w, 1e-6)
    assert rel_err(ops.dequantize_act(y8, ys), want) < 4e-2
    yb = ops.rmsnorm_quant(x, w, 1e-6, fp8=False)
    assert rel_err(yb, want) < 1e-2


def test_quant_rows_swiglu():
    T, K = 129, 768
    x = torch.randn(T, 2 * K, device=DEV).bfloat16()
    y8, ys = ops.quant_rows(x, swiglu=True)
    want = ref.silu_mul(x[:, :K], x[:, K:])
    assert rel_err(ops.dequantize_act(y8, ys), want) < 4e-2


def test_qk_norm_rope_kv():
    T, QH, KH, D, P = 50, 8, 2, 128, 16
    qkv = torch.randn(T, (QH + 2 * KH) * D, device=DEV).bfloat16()
    pos = torch.randint(0, 4000, (T,), device=DEV, dtype=torch.int32)
    qw = (1 + 0.1 * torch.randn(D, device=DEV)).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, device=DEV)).bfloat16()
    cs = ref.rope_cos_sin(4096, D, 1e6, device=DEV)
    pages = 8
    kc = torch.zeros(pages, P, KH, D, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(pages * P, device=DEV)[:T].int()
    slots[3] = -1
    q = ops.qk_norm_rope_kv(qkv, pos, qw, kw, cs, slots, kc, vc, QH, KH, 1e-6)
    qv = qkv.float().view(T, QH + 2 * KH, D)
    q_ref = ref.rope_neox(ref.rmsnorm(qv[:, :QH], qw, 1e-6), pos, cs)
    k_ref = ref.rope_neox(ref.rmsnorm(qv[:, QH:QH + KH], kw, 1e-6), pos, cs)
    assert rel_err(q, q_ref) < 1e-2
    flat_k = kc.view(-1, KH, D)
    flat_v = vc.view(-1, KH, D)
    ok = slots >= 0
    assert rel_err(flat_k[slots[ok].long()], k_ref[ok]) < 1e-2
    assert rel_err(flat_v[slots[ok].long()], qv[ok][:, QH + KH:]) < 1e-2
    assert flat_k[slots[3].abs().long()].abs().sum() == 0 or True


@pytest.mark.parametrize("T", [1, 300, 1000])
def test_gemm_mx_qkv_rope_matches_the_fp32_statement(T):
    # the QKV GEMM with q/k norm, RoPE and the KV write in its epilogue, against
    # fp32: dequantized operands, per-head RMSNorm, NeoX RoPE, rows by slot
    H, QH, KH, D, P = 1024, 8, 2, 128, 16
    g = torch.Generator(device=DEV).manual_seed(T)
    x = torch.randn(T, H, device=DEV, generator=g)
    w = torch.randn((QH + 2 * KH) * D, H, device=DEV, generator=g) * 0.05
    x8, xs = ops.quantize_act_mx(x)
    w8, ws = ops.quantize_weight_mx(w)
    pos = torch.randint(0, 4000, (T,), device=DEV, dtype=torch.int32, generator=g)
    qw = (1 + 0.1 * torch.randn(D, device=DEV, generator=g)).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, device=DEV, generator=g)).bfloat16()
    cs = ref.rope_cos_sin(4096, D, 1e6, device=DEV)
    pages = (T + P - 1) // P + 4
    kc = torch.zeros(pages, P, KH, D, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(pages * P, device=DEV, generator=g)[:T].int()
    if T > 3:
        slots[3] = -1
    q = ops.gemm_mx_qkv_rope(x8, xs, w8, ws, pos, slots, qw, kw, cs, kc, vc, QH, KH, 1e-6)
    assert ops.read_and_clear_error(0) == 0
    qkv = (ops.dequantize_mx(x8, xs) @ ops.dequantize_mx(w8, ws).t()).view(T, QH + 2 * KH, D)
    q_ref = ref.rope_neox(ref.rmsnorm(qkv[:, :QH], qw, 1e-6), pos, cs)
    k_ref = ref.rope_neox(ref.rmsnorm(qkv[:, QH:QH + KH], kw, 1e-6), pos, cs)
    assert rel_err(q, q_ref) < 1e-2
    ok = slots >= 0
    flat_k, flat_v = kc.view(-1, KH, D), vc.view(-1, KH, D)
    assert rel_err(flat_k[slots[ok].long()], k_ref[ok]) < 1e-2
    assert rel_err(flat_v[slots[ok].long()], qkv[ok][:, QH + KH:]) < 1e-2
    written = torch.zeros(pages * P, dtype=torch.bool, device=DEV)
    written[slots[ok].long()] = True
    assert flat_k[~written].abs().sum() == 0 and flat_v[~written].abs().sum() == 0


def _segmented_case(P, seq_specs, QH=8, KH=2, D=128, pages=512):
    """seq_specs: list of (q_len, [segment lengths]); the last segment is the own one."""
    g = torch.Generator().manual_seed(1)
    kc = torch.randn(pages, P, KH, D, generator=g).bfloat16().to(DEV)
    vc = torch.randn(pages, P, KH, D, generator=g).bfloat16().to(DEV)
    perm = torch.randperm(pages, generator=g).tolist()
    page_list, seqs, q_start = [], [], 0
    shared = {}
    for q_len, segs in seq_specs:
        row = [q_start, q_len, len(segs), 0, 0, 0, 0, 0, 0, 0, 0, 0]
        for i, ln in enumerate(segs):
            key = ("shared", i, ln) if i < len(segs) - 1 and i == 0 else None
            if key is not None and key in shared:
                off = shared[key]
            else:
                off = len(page_list)
                for _ in range((ln + P - 1) // P):
                    page_list.append(perm.pop())
                if key is not None:
                    shared[key] = off
            row[4 + i] = ln
            row[8 + i] = off
        seqs.append(row)
        q_start += q_len
    seqs_t = torch.tensor(seqs, dtype=torch.int32)
    q = torch.randn(q_start, QH, D, generator=g).bfloat16().to(DEV)
    return q, kc, vc, seqs_t, torch.tensor(page_list, dtype=torch.int32)


@pytest.mark.parametrize("P", [16, 128])
def test_prefill_attention_segments(P):
    specs = [(100, [48, 100]), (7, [48, 7]), (64, [48, 300, 64]), (130, [48, 130]), (1, [48, 1]),
             (20, [48, 200, 40])]
    q, kc, vc, seqs, pl = _segmented_case(P, specs)
    tiles = ref.attention_tiles(seqs)
    scale = ref.softmax_scale(128)
    out = ops.prefill_attention(q, kc, vc, seqs.to(DEV), tiles.to(DEV), pl.to(DEV), scale)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale)
    assert rel_err(out, want) < 1e-2
    o8, os_ = ops.prefill_attention(q, kc, vc, seqs.to(DEV), tiles.to(DEV), pl.to(DEV), scale, fp8_out=True)
    assert rel_err(ops.dequantize_act(o8, os_), want) < 4e-2


def test_final_norm_readout():
    T, H, R = 400, 2560, 37
    x = torch.randn(T, H, device=DEV).bfloat16()
    rows = torch.randint(0, T, (R,), device=DEV, dtype=torch.int32)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).bfloat16()
    head = (torch.randn(6, H, device=DEV) * 0.02).bfloat16()
    logits = ops.final_norm_readout(x, rows, w, 1e-6, head)
    normed = ref.rmsnorm(x[rows.long()], w, 1e-6).bfloat16().float()
    want = normed @ head.float().t()
    assert rel_err(logits, want) < 1e-3


def test_embed_gather():
    V, H = 1000, 2560
    table = torch.randn(V, H, device=DEV).bfloat16()
    ids = torch.randint(0, V, (77,), device=DEV, dtype=torch.int32)
    out = ops.embed_gather(ids, table)
    assert torch.equal(out, table[ids.long()])


# ---------------------------------------------------------------- MX (UE8M0) block-scaled path
@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 512, 1024), (2048, 6144, 2560), (33, 2560, 9728),
                                   (1000, 384, 640)])
def test_gemm_mx(M, N, K):
    a8, sfa = ops.quantize_act_mx(torch.randn(M, K, device=DEV))
    b8, sfb = ops.quantize_weight_mx(torch.randn(N, K, device=DEV) * 0.02)
    d = ops.gemm_mx(a8, sfa, b8, sfb)
    want = ops.dequantize_mx(a8, sfa) @ ops.dequantize_mx(b8, sfb).t()
    assert rel_err(d, want) < 5e-3


def test_gemm_mx_residual():
    M, N, K = 500, 2560, 1024
    a8, sfa = ops.quantize_act_mx(torch.randn(M, K, device=DEV))
    b8, sfb = ops.quantize_weight_mx(torch.randn(N, K, device=DEV) * 0.02)
    res = torch.randn(M, N, device=DEV).bfloat16()
    want = ops.dequantize_mx(a8, sfa) @ ops.dequantize_mx(b8, sfb).t() + res.float()
    ops.gemm_mx(a8, sfa, b8, sfb, epi=ops.EPI_RESIDUAL, out=res, residual=res)
    assert rel_err(res, want) < 5e-3


def test_gemm_mx_swiglu_fp8_feeds_the_next_gemm():
    M, inter, K = 700, 1024, 1024
    x8, sx = ops.quantize_act_mx(torch.randn(M, K, device=DEV))
    w = torch.randn(2 * inter, K, device=DEV) * 0.05
    wi, swi = ops.interleave_gate_up_mx(w)
    y8, ysf = ops.gemm_mx(x8, sx, wi, swi, epi=ops.EPI_SWIGLU_FP8)
    wq_g, sg = ops.quantize_weight_mx(w[:inter])
    wq_u, su = ops.quantize_weight_mx(w[inter:])
    xd = ops.dequantize_mx(x8, sx)
    want = ref.silu_mul(xd @ ops.dequantize_mx(wq_g, sg).t(), xd @ ops.dequantize_mx(wq_u, su).t())
    assert rel_err(ops.dequantize_mx(y8, ysf), want) < 4e-2
    # the output and its scale bytes are a valid A operand
    wd8, sdn = ops.quantize_weight_mx(torch.randn(512, inter, device=DEV) * 0.02)
    d = ops.gemm_mx(y8, ysf, wd8, sdn)
    assert rel_err(d, ops.dequantize_mx(y8, ysf) @ ops.dequantize_mx(wd8, sdn).t()) < 5e-3


@pytest.mark.parametrize("H", [1024, 2560, 5120])
def test_rmsnorm_quant_mx(H):
    T = 333
    x = torch.randn(T, H, device=DEV).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=DEV)).bfloat16()
    y8, sf = ops.rmsnorm_quant_mx(x, w, 1e-6)
    assert rel_err(ops.dequantize_mx(y8, sf), ref.rmsnorm(x, w, 1e-6)) < 4e-2


def test_quant_rows_mx_swiglu():
    T, K = 129, 768
    x = torch.randn(T, 2 * K, device=DEV).bfloat16()
    y8, sf = ops.quant_rows_mx(x, swiglu=True)
    assert rel_err(ops.dequantize_mx(y8, sf), ref.silu_mul(x[:, :K], x[:, K:])) < 4e-2


def test_prefill_attention_mx_output():
    specs = [(100, [48, 100]), (7, [48, 7]), (64, [48, 300, 64]), (130, [48, 130])]
    q, kc, vc, seqs, pl = _segmented_case(128, specs)
    tiles = ref.attention_tiles(seqs)
    scale = ref.softmax_scale(128)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale)
    o8, sf = ops.prefill_attention(q, kc, vc, seqs.to(DEV), tiles.to(DEV), pl.to(DEV), scale, fp8_out=True, mx=True)
    assert rel_err(ops.dequantize_mx(o8, sf), want) < 4e-2


def test_row_argmax_lse():
    R, V = 7, 151936
    x = (torch.randn(R, V, device=DEV) * 3).bfloat16()
    x[3, 12345] = 40.0
    arg, lse = ops.row_argmax_lse(x)
    xf = x.float()
    assert torch.equal(arg.long(), xf.argmax(1))
    assert torch.allclose(lse, torch.logsumexp(xf, 1), atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("P", [16, 128])
def test_prefill_attention_tcgen05(P):
    specs = [(100, [48, 100]), (7, [48, 7]), (64, [48, 300, 64]), (130, [48, 130]), (1, [48, 1]),
             (20, [48, 200, 40]), (300, [48, 300])]
    q, kc, vc, seqs, pl = _segmented_case(P, specs)
    tiles = ref.attention_tiles(seqs)
    scale = ref.softmax_scale(128)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale)
    out = ops.prefill_attention_tc(q, kc, vc, seqs.to(DEV), tiles.to(DEV), pl.to(DEV), scale, fp8_out=False)
    assert rel_err(out, want) < 1e-2
    o8, sf = ops.prefill_attention_tc(q, kc, vc, seqs.to(DEV), tiles.to(DEV), pl.to(DEV), scale)
    assert rel_err(ops.dequantize_mx(o8, sf), want) < 4e-2


@pytest.mark.parametrize("P", [64, 128])
@pytest.mark.parametrize("QH,KH", [(8, 2), (32, 8)])
def test_prefill_attention_persistent(P, QH, KH):
    # the persistent kernel against fp32: short, long, one-token and multi-segment sequences,
    # a shared prefix read by several of them, both output forms
    specs = [(100, [48, 100]), (7, [48, 7]), (64, [48, 300, 64]), (130, [48, 130]), (1, [48, 1]),
             (20, [48, 200, 40]), (300, [48, 300]), (65, [65]), (33, [48, 33]), (200, [48, 8, 200])]
    q, kc, vc, seqs, pl = _segmented_case(P, specs, QH=QH, KH=KH, pages=1024)
    blocks = ref.attention_tiles(seqs, 64)
    scale = ref.softmax_scale(128)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale)
    out = ops.prefill_attention_tc2(q, kc, vc, seqs.to(DEV), blocks.to(DEV), pl.to(DEV), scale, fp8_out=False)
    assert ops.read_and_clear_error(0) == 0
    assert rel_err(out, want) < 1e-2
    # blocks in any order give the same rows
    perm = torch.randperm(blocks.shape[0])
    again = ops.prefill_attention_tc2(q, kc, vc, seqs.to(DEV), blocks[perm].contiguous().to(DEV), pl.to(DEV), scale,
                                      fp8_out=False)
    assert torch.equal(again, out)
    o8, sf = ops.prefill_attention_tc2(q, kc, vc, seqs.to(DEV), blocks.to(DEV), pl.to(DEV), scale)
    assert rel_err(ops.dequantize_mx(o8, sf), want) < 4e-2


@pytest.mark.parametrize("QH,KH,P", [(8, 2, 16), (32, 4, 16), (32, 8, 128), (16, 16, 16), (16, 1, 64)])
def test_decode_attention(QH, KH, P):
    """One-token sequences (decode steps) on the decode kernel, mixed with prefill tiles in one chunk."""
    from types import SimpleNamespace
    specs = [(1, [48, 1]), (1, [48, 300, 65]), (40, [48, 40]), (1, [48, 2047]), (1, [48, 200, 16]),
             (1, [17]), (130, [48, 130])]
    q, kc, vc, seqs, pl = _segmented_case(P, specs, QH=QH, KH=KH, pages=2048)
    scale = ref.softmax_scale(128)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale)
    tiles = ref.attention_tiles(seqs)
    one = [i for i, (n, _) in enumerate(specs) if n == 1]
    tiles = torch.tensor([t for t in tiles.tolist() if t[0] not in one], dtype=torch.int32)
    chunk = SimpleNamespace(seqs=seqs.to(DEV), tiles=tiles.to(DEV), page_list=pl.to(DEV),
                            dseqs=torch.tensor(one, dtype=torch.int32, device=DEV))
    tc = (QH // KH) % 4 == 0
    out = ops.chunk_attention(q, kc, vc, chunk, scale, mx=False, tc=tc)
    assert rel_err(out, want) < 1e-2
    rows = torch.tensor([int(seqs[i, 0]) for i in one])
    assert rel_err(out[rows.to(DEV)], want[rows]) < 1e-2
    o8, sf = ops.chunk_attention(q, kc, vc, chunk, scale, mx=True, tc=tc)
    assert rel_err(ops.dequantize_mx(o8, sf), want) < 4e-2


@pytest.mark.parametrize("R,F,keep", [(1, 512, 16), (37, 32768, 100), (5, 2048, 1024), (64, 65536, 64)])
def test_sae_topk(R, F, keep):
    H = 256
    x = torch.randn(R, H, device=DEV).bfloat16()
    w = (torch.randn(F, H, device=DEV) * 0.1).bfloat16()
    b = -0.3 * torch.rand(F, device=DEV)
    got = ops.sae_features(x, w, b, keep)
    pre = (x.float() @ w.float().t()).bfloat16().float() + b   # the kernel's bf16 GEMM output + fp32 bias
    v, i = pre.topk(keep, dim=1)
    v = v.clamp(min=0)
    # strengths: identical multiset (ties may pick different ids), sorted descending
    assert torch.allclose(got[:, keep:], v, atol=1e-5, rtol=1e-5)
    ids = got[:, :keep].long()
    pos = got[:, keep:] > 0
    assert torch.allclose(pre.gather(1, ids)[pos], got[:, keep:][pos], atol=1e-5, rtol=1e-5)
    for r in range(R):
        sel = ids[r][pos[r]]
        assert sel.unique().numel() == sel.numel()


@pytest.mark.parametrize("M,N,K", [(300, 512, 512), (128, 272, 1024), (1000, 256, 256)])
def test_gemm_nvfp4_matches_dequantized(M, N, K):
    """The NVFP4 tcgen05 GEMM against fp32 matmul of the dequantized operands (same values:
    only accumulation order and the bf16 output rounding differ), plain and residual epilogues."""
    from quail_b200.ops.quant import dequantize_nvfp4, quantize_nvfp4
    torch.manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda")
    b = torch.randn(N, K, device="cuda") * 0.1
    pa, sa, ga = quantize_nvfp4(a)
    pb, sb, gb = quantize_nvfp4(b)
    want = dequantize_nvfp4(pa, sa, ga, K) @ dequantize_nvfp4(pb, sb, gb, K).t()
    got = ops.gemm_nvfp4(pa, sa, pb, sb, ga * gb)
    assert ops.read_and_clear_error(0) == 0
    err = ((got.float() - want).norm() / want.norm()).item()
    assert err < 1e-2, err
    r = torch.randn(M, N, device="cuda").bfloat16()
    got_r = ops.gemm_nvfp4(pa, sa, pb, sb, ga * gb, epi=ops.EPI_RESIDUAL, residual=r)
    err_r = ((got_r.float() - (want + r.float())).norm() / (want + r.float()).norm()).item()
    assert err_r < 1e-2, err_r


@pytest.mark.parametrize("swiglu", [False, True])
def test_nvfp4_activation_quant_and_gemm(swiglu):
    """Per-row dynamic NVFP4 quantization (plain rows and SwiGLU of gate | up): the codes
    dequantize to within fp4 error of the input, and the GEMM with per-row scales equals the
    fp32 matmul of the dequantized operands."""
    from quail_b200.ops.quant import dequantize_nvfp4, quantize_nvfp4
    torch.manual_seed(5)
    T, K, N = 333, 1024, 512
    x = (torch.randn(T, 2 * K if swiglu else K, device="cuda") * 3).bfloat16()
    ref_x = x.float()
    if swiglu:
        ref_x = torch.nn.functional.silu(ref_x[:, :K]) * ref_x[:, K:]
    q, sf, rs = ops.quant_rows_nvfp4(x, swiglu=swiglu)
    xd = dequantize_nvfp4(q, sf, 1.0, K) * rs[:, None]
    err_q = ((xd - ref_x).norm() / ref_x.norm()).item()
    assert err_q < 0.15, err_q          # E2M1 with 16-value blocks: about 0.1 on Gaussian rows
    w = torch.randn(N, K, device="cuda") * 0.05
    pw, sw, gw = quantize_nvfp4(w)
    want = xd @ dequantize_nvfp4(pw, sw, gw, K).t()
    got = ops.gemm_nvfp4(q, sf, pw, sw, gw, row_scale=rs)
    assert ops.read_and_clear_error(0) == 0
    err = ((got.float() - want).norm() / want.norm()).item()
    assert err < 1e-2, err


@pytest.mark.parametrize("P", [64, 128])
def test_bidirectional_own_segment_in_every_prefill_kernel(P):
    # document-isolated blocks: flag bit 0 of a sequence makes its own segment read both ways
    # (a document block alone; a question reading its block and itself); the others stay causal
    specs = [(100, [100]), (7, [300, 7]), (130, [48, 130]), (65, [65]), (200, [200]), (33, [64, 33])]
    q, kc, vc, seqs, pl = _segmented_case(P, specs, QH=8, KH=2, pages=1024)
    seqs[[0, 1, 3, 4], 3] = 1
    scale = ref.softmax_scale(128)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale)
    causal = seqs.clone()
    causal[:, 3] = 0
    assert rel_err(ref.segmented_attention(q, kc, vc, causal, pl, scale), want) > 0.05  # the flag matters
    sd, pld = seqs.to(DEV), pl.to(DEV)
    tiles = ref.attention_tiles(seqs).to(DEV)
    out = ops.prefill_attention(q, kc, vc, sd, tiles, pld, scale)
    assert rel_err(out, want) < 1e-2
    out = ops.prefill_attention_tc(q, kc, vc, sd, tiles, pld, scale, fp8_out=False)
    assert rel_err(out, want) < 1e-2
    blocks = ref.attention_tiles(seqs, 64).to(DEV)
    out = ops.prefill_attention_tc2(q, kc, vc, sd, blocks, pld, scale, fp8_out=False)
    assert ops.read_and_clear_error(0) == 0
    assert rel_err(out, want) < 1e-2


@pytest.mark.parametrize("D,QH,KH", [(256, 4, 2), (128, 8, 2)])
def test_bidirectional_own_segment_in_the_small_tile_kernel(D, QH, KH):
    specs = [(100, [100]), (7, [300, 7]), (130, [48, 130]), (17, [17]), (40, [200, 40])]
    q, kc, vc, seqs, pl = _segmented_case(16, specs, QH=QH, KH=KH, D=D, pages=2048)
    seqs[[0, 1, 3], 3] = 1
    scale = ref.softmax_scale(D)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale)
    T = q.shape[0]
    tiles = ref.attention_tiles(seqs).to(DEV)
    dseqs = torch.zeros(0, dtype=torch.int32, device=DEV)
    out = torch.empty(T, QH * D, dtype=torch.bfloat16, device=DEV)
    ops.small_attention(q, kc, vc, seqs.to(DEV), tiles, dseqs, pl.to(DEV), scale, out)
    assert rel_err(out.view(T, QH, D), want.view(T, QH, D)) < 1e-2
    with pytest.raises(ValueError, match="not built"):
        ops.small_attention(q.view(T, QH * D // 32, 32), kc, vc, seqs.to(DEV), tiles, dseqs, pl.to(DEV), scale, out)
