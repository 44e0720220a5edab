"""Thin wrappers that allocate outputs and call the compiled kernels."""

from __future__ import annotations

import importlib

import torch

_C = None
_IMPORT_ERROR: Exception | None = None
try:
    _C = importlib.import_module("quail_b200._C")
except Exception as exc:  # noqa: BLE001 - surfaced by native()
    _IMPORT_ERROR = exc

# kernels launched through these wrappers (bench.py reports the count per timed region)
_LAUNCHES = [0]


def launch_count() -> int:
    return _LAUNCHES[0]


def count_launch(n: int = 1) -> None:
    _LAUNCHES[0] += n


EPI_BF16 = 0
EPI_RESIDUAL = 1
EPI_SWIGLU_FP8 = 2
EPI_SWIGLU_BF16 = 3
EPI_GEGLU_BF16 = 6
EPI_GEGLU_FP8 = 7
EPI_RESIDUAL_MX = 5


def kernels_available() -> bool:
    return _C is not None


def native():
    """The compiled extension; raises if it was not built."""
    if _C is None:
        raise RuntimeError(
            "quail_b200._C is not built (run `python setup.py build_ext --inplace`): "
            f"{_IMPORT_ERROR}")
    return _C


def gemm(a: torch.Tensor, b: torch.Tensor, *, sa: torch.Tensor | None = None,
         sb: torch.Tensor | None = None, sb_gran: int = 128, epi: int = EPI_BF16,
         out: torch.Tensor | None = None, out_scale: torch.Tensor | None = None,
         residual: torch.Tensor | None = None, bn: int = 256):
    """D = A . B^T on the tcgen05 GEMM.

    A [M, K] and B [N, K] are both bf16, or both e4m3 with `sa` [K/128, >=M]
    (one fp32 scale per token and 128-wide K group) and `sb`
    [ceil(N/sb_gran), K/128]. Epilogues: EPI_BF16 -> [M, N] bf16;
    EPI_RESIDUAL -> out = acc + residual (out may be the residual itself);
    EPI_SWIGLU_BF16 -> [M, N/2] bf16 of silu(gate) * up over a gate/up
    interleaved B (EPI_GEGLU_BF16: gelu_tanh(gate) * up; bf16 operands only);
    EPI_SWIGLU_FP8 -> ([M, N/2] e4m3, [N/256, M] scales).
    """
    C = native()
    M, N = a.shape[0], b.shape[0]
    if epi == EPI_SWIGLU_FP8:
        if out is None:
            out = torch.empty(M, N // 2, dtype=torch.float8_e4m3fn, device=a.device)
        if out_scale is None:
            out_scale = torch.empty(N // 256, M, dtype=torch.float32, device=a.device)
        count_launch()
        C.gemm(a, b, sa, sb, sb_gran, epi, out, out_scale, None, bn)
        return out, out_scale
    if out is None:
        width = N // 2 if epi in (EPI_SWIGLU_BF16, EPI_GEGLU_BF16) else N
        out = torch.empty(M, width, dtype=torch.bfloat16, device=a.device)
    count_launch()
    C.gemm(a, b, sa, sb, sb_gran, epi, out, None, residual, bn)
    return out


def sf_bytes(rows: int, K: int) -> int:
    """Bytes of MX scale atoms for a [rows, K] e4m3 matrix."""
    return -(-rows // 128) * (K // 128) * 512


def gemm_mx(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, *, epi: int = EPI_BF16,
            out: torch.Tensor | None = None, out_sf: torch.Tensor | None = None,
            residual: torch.Tensor | None = None, row_ss: torch.Tensor | None = None, eps: float = 1e-6,
            xq: torch.Tensor | None = None, xq_sf: torch.Tensor | None = None, ss_out: torch.Tensor | None = None):
    """D = A . B^T with UE8M0 block scales on the tcgen05 block-scaled MMA.

    A [M, K], B [N, K] e4m3; sfa / sfb their scale bytes in the MX atom
    layout (quail_b200.ops.quant.pack_sf_atoms). EPI_SWIGLU_FP8 returns
    (e4m3 [M, N/2], its scale bytes) ready to be the next GEMM's A.

    row_ss [M, parts] (partial sums of squares of A's unnormalized rows): the
    rows are RMS-normalized in the epilogue (rsqrt(sum / K + eps)), for an A
    that came out of EPI_RESIDUAL_MX or quant_mx_ss and a B with the norm
    weight folded in. EPI_RESIDUAL_MX: out = acc + residual (bf16), and out as
    e4m3 + MX scales into xq / xq_sf, with each row's sums of squares per 128
    columns into ss_out [M, N / 128].
    """
    C = native()
    M, N = a.shape[0], b.shape[0]
    count_launch()
    if epi in (EPI_SWIGLU_FP8, EPI_GEGLU_FP8):
        if out is None:
            out = torch.empty(M, N // 2, dtype=torch.float8_e4m3fn, device=a.device)
        if out_sf is None:
            out_sf = torch.empty(sf_bytes(M, N // 2), dtype=torch.uint8, device=a.device)
        C.gemm_mx(a, sfa, b, sfb, epi, out, out_sf, None, row_ss, eps, None, None, None)
        return out, out_sf
    if out is None:
        out = torch.empty(M, N // 2 if epi == EPI_SWIGLU_BF16 else N, dtype=torch.bfloat16, device=a.device)
    C.gemm_mx(a, sfa, b, sfb, epi, out, None, residual, row_ss, eps, xq, xq_sf, ss_out)
    return out


def row_rinv(parts: torch.Tensor, K: int, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """1 / rms per row, [M] fp32, from [M, n] partial sums of squares over K columns."""
    if out is None:
        out = torch.empty(parts.shape[0], dtype=torch.float32, device=parts.device)
    count_launch()
    native().row_rinv(parts, K, eps, out)
    return out


def quant_mx_ss(x: torch.Tensor, *, out=None, out_sf=None, ss=None, rows: int | None = None):
    """bf16 rows -> (e4m3 rows, MX scale bytes, per-row sum of squares): a GEMM input whose
    RMSNorm the GEMM applies (gemm_mx(row_ss=...))."""
    T = x.shape[0] if rows is None else rows
    H = x.shape[1]
    _check_hidden(H, "quant_mx_ss")
    out = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=x.device) if out is None else out
    out_sf = torch.empty(sf_bytes(T, H), dtype=torch.uint8, device=x.device) if out_sf is None else out_sf
    ss = torch.empty(T, 1, dtype=torch.float32, device=x.device) if ss is None else ss
    count_launch()
    native().quant_mx_ss(x, out, out_sf, ss, T)
    return out, out_sf, ss


def gemm_mx_qkv_rope(x8, xs, wqkv, sqkv, positions, slots, q_norm_w, k_norm_w, cos_sin, k_cache, v_cache,
                     num_q_heads: int, num_kv_heads: int, eps: float, *, norm_qk: bool = True, q_out=None,
                     row_ss=None):
    """The fp8 QKV projection with per-head q/k RMSNorm, NeoX RoPE and the paged KV write
    fused into its epilogue (K1 + K4 in one kernel). Returns q [T, QH, 128] bf16."""
    C = native()
    T = x8.shape[0]
    if q_out is None:
        q_out = torch.empty(T, num_q_heads, 128, dtype=torch.bfloat16, device=x8.device)
    count_launch()
    C.gemm_mx_qkv_rope(x8, xs, wqkv, sqkv, positions, slots, q_norm_w, k_norm_w, cos_sin, q_out, k_cache, v_cache,
                       num_q_heads, num_kv_heads, eps, norm_qk, row_ss)
    return q_out


def quant_rows_nvfp4(x: torch.Tensor, *, swiglu: bool = False):
    """bf16 rows (or silu(gate) * up of [T, 2K] gate | up) -> (packed E2M1 [T, K/2], UE4M3 block-scale
    atoms, fp32 per-row scale [T]) for gemm_nvfp4's A side."""
    T = x.shape[0]
    K = x.shape[1] // 2 if swiglu else x.shape[1]
    q = torch.empty(T, K // 2, dtype=torch.uint8, device=x.device)
    sf = torch.empty(-(-T // 128) * (K // 64) * 512, dtype=torch.uint8, device=x.device)
    rs = torch.empty(T, dtype=torch.float32, device=x.device)
    count_launch()
    native().nvfp4_quant_rows(x, swiglu, q, sf, rs)
    return q, sf, rs


def gemm_nvfp4(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: float, *,
               epi: int = EPI_BF16, out: torch.Tensor | None = None, residual: torch.Tensor | None = None,
               row_scale: torch.Tensor | None = None):
    """D = alpha . A . B^T on the tcgen05 NVFP4 MMA (kind::mxf4nvf4, 16-value UE4M3 block scales).

    A [M, K/2], B [N, K/2] packed E2M1 (uint8); sfa / sfb their block-scale
    atoms (quail_b200.ops.quant.quantize_nvfp4); alpha the product of the two
    global scales, row_scale an optional per-row scale of A (quant_rows_nvfp4's).
    EPI_BF16 or EPI_RESIDUAL (out = acc + residual).
    """
    M, N = a.shape[0], b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    count_launch()
    native().gemm_nvfp4(a, sfa, b, sfb, float(alpha), epi, out, residual, row_scale)
    return out


def rmsnorm_quant_mx(x: torch.Tensor, w: torch.Tensor, eps: float, *, out=None, out_sf=None, rows=None):
    """RMSNorm -> (e4m3 [T, H], UE8M0 scale bytes, one per 32 columns)."""
    T = x.shape[0] if rows is None else rows
    H = x.shape[1]
    _check_hidden(H, "rmsnorm_quant_mx")
    if out is None:
        out = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=x.device)
    if out_sf is None:
        out_sf = torch.empty(sf_bytes(T, H), dtype=torch.uint8, device=x.device)
    count_launch()
    native().rmsnorm_quant_mx(x, w, eps, out, out_sf, T)
    return out, out_sf


def quant_rows_mx(x: torch.Tensor, *, swiglu: bool = False, rows: int | None = None):
    T = x.shape[0] if rows is None else rows
    K = x.shape[1] // 2 if swiglu else x.shape[1]
    y = torch.empty(T, K, dtype=torch.float8_e4m3fn, device=x.device)
    sf = torch.empty(sf_bytes(T, K), dtype=torch.uint8, device=x.device)
    count_launch()
    native().quant_rows_mx(x, swiglu, y, sf, T)
    return y, sf


def embed_gather(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None):
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=torch.bfloat16, device=ids.device)
    count_launch()
    native().embed_gather(ids, table, out)
    return out


# hidden sizes the row kernels (RMSNorm + quantization, final norm readout) are instantiated for
NORM_HIDDEN = frozenset({256, 512, 1024, 2048, 2560, 2816, 4096, 5120})


def _check_hidden(H: int, what: str) -> None:
    """Refuse a hidden size the native row kernels are not built for here, in Python: the native
    check would raise inside the extension instead."""
    if H not in NORM_HIDDEN:
        raise ValueError(f"{what}: hidden size {H} is not built; built: {sorted(NORM_HIDDEN)}")


def rmsnorm_quant(x: torch.Tensor, w: torch.Tensor, eps: float, *, fp8: bool = True,
                  out=None, out_scale=None, rows: int | None = None):
    """RMSNorm of x's first `rows` rows -> (e4m3 [T, H], scales [H/128, T]) or bf16."""
    T = x.shape[0] if rows is None else rows
    H = x.shape[1]
    _check_hidden(H, "rmsnorm_quant")
    if fp8:
        if out is None:
            out = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=x.device)
        if out_scale is None:
            out_scale = torch.empty(H // 128, T, dtype=torch.float32, device=x.device)
        count_launch()
        native().rmsnorm_quant(x, w, eps, out, out_scale, None, T)
        return out, out_scale
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    count_launch()
    native().rmsnorm_quant(x, w, eps, None, None, out, T)
    return out


def quant_rows(x: torch.Tensor, *, swiglu: bool = False, fp8: bool = True, rows: int | None = None):
    """bf16 rows -> e4m3 + 1x128 scales (optionally SwiGLU of [gate | up] first)."""
    T = x.shape[0] if rows is None else rows
    K = x.shape[1] // 2 if swiglu else x.shape[1]
    if fp8:
        y = torch.empty(T, K, dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.empty(K // 128, T, dtype=torch.float32, device=x.device)
        count_launch()
        native().quant_rows(x, swiglu, y, s, None, T)
        return y, s
    y = torch.empty(T, K, dtype=torch.bfloat16, device=x.device)
    count_launch()
    native().quant_rows(x, swiglu, None, None, y, T)
    return y


def qk_norm_rope_kv(qkv, positions, q_norm_w, k_norm_w, cos_sin, slots, k_cache, v_cache,
                    num_q_heads: int, num_kv_heads: int, eps: float, *, norm_qk: bool = True,
                    q_out=None, rows: int | None = None):
    """Per-head q/k RMSNorm + NeoX RoPE; q -> [T, QH, 128]; k, v -> cache[slot]."""
    T = qkv.shape[0] if rows is None else rows
    if q_out is None:
        q_out = torch.empty(T, num_q_heads, 128, dtype=torch.bfloat16, device=qkv.device)
    count_launch()
    native().qk_norm_rope_kv(qkv, positions, q_norm_w, k_norm_w, cos_sin, slots, q_out, k_cache,
                             v_cache, num_q_heads, num_kv_heads, eps, norm_qk, T)
    return q_out


def prefill_attention(q, k_cache, v_cache, seqs, tiles, page_list, softmax_scale: float, *,
                      fp8_out: bool = False, mx: bool = False, out=None, out_scale=None):
    """Segmented paged attention (see csrc/attention.cu) -> [T, QH*128].

    fp8_out: e4m3 + one fp32 scale per (token, head) [QH, T]; with mx, e4m3 +
    UE8M0 scale bytes per 32 values in the MX atom layout (the o_proj A input).
    """
    T, QH = q.shape[0], q.shape[1]
    if fp8_out and mx:
        if out is None:
            out = torch.empty(T, QH * 128, dtype=torch.float8_e4m3fn, device=q.device)
        if out_scale is None:
            out_scale = torch.empty(sf_bytes(T, QH * 128), dtype=torch.uint8, device=q.device)
        count_launch()
        native().prefill_attention(q, k_cache, v_cache, seqs, tiles, page_list, softmax_scale, out, out_scale)
        return out, out_scale
    if fp8_out:
        if out is None:
            out = torch.empty(T, QH * 128, dtype=torch.float8_e4m3fn, device=q.device)
        if out_scale is None:
            out_scale = torch.empty(QH, T, dtype=torch.float32, device=q.device)
        count_launch()
        native().prefill_attention(q, k_cache, v_cache, seqs, tiles, page_list, softmax_scale,
                                   out, out_scale)
        return out, out_scale
    if out is None:
        out = torch.empty(T, QH * 128, dtype=torch.bfloat16, device=q.device)
    count_launch()
    native().prefill_attention(q, k_cache, v_cache, seqs, tiles, page_list, softmax_scale, out, None)
    return out


def prefill_attention_tc(q, k_cache, v_cache, seqs, tiles, page_list, softmax_scale: float, *,
                         fp8_out: bool = True, out=None, out_scale=None):
    """The tcgen05/TMEM attention kernel (needs 4 q heads per KV head): bf16 or e4m3 + MX scale bytes."""
    T, QH = q.shape[0], q.shape[1]
    if out is None:
        out = torch.empty(T, QH * 128, dtype=torch.float8_e4m3fn if fp8_out else torch.bfloat16, device=q.device)
    if fp8_out and out_scale is None:
        out_scale = torch.empty(sf_bytes(T, QH * 128), dtype=torch.uint8, device=q.device)
    count_launch()
    native().prefill_attention_tc(q, k_cache, v_cache, seqs, tiles, page_list, softmax_scale, out,
                                  out_scale if fp8_out else None)
    return (out, out_scale) if fp8_out else out


def decode_attention(q, k_cache, v_cache, seqs, dseqs, page_list, softmax_scale: float, out, out_scale=None):
    """One-query-token sequences (decode steps): csrc/attention_decode.cu, into `out` (bf16 or e4m3 + atoms)."""
    if dseqs.numel() == 0:
        return
    count_launch()
    native().decode_attention(q, k_cache, v_cache, seqs, dseqs, page_list, softmax_scale, out, out_scale)


def prefill_attention_tc2(q, k_cache, v_cache, seqs, blocks, page_list, softmax_scale: float, *,
                          fp8_out: bool = True, out=None, out_scale=None, lse=None):
    """The persistent tcgen05 attention (csrc/attention_tc2.cu) over 64-token query blocks.

    blocks [m, 2] int32: (sequence, first query token) per 64-token block
    (`ops.reference.attention_tiles(seqs, 64)` or a chunk's `blocks`); pages
    hold a multiple of 64 tokens. Returns bf16 [T, QH*128], or with fp8_out
    (e4m3, UE8M0 scale bytes in the MX atom layout). With a bf16 out, `lse`
    (fp32 [T, QH]) receives each row's log-sum-exp for a later merge.
    """
    T, QH = q.shape[0], q.shape[1]
    if out is None:
        out = torch.empty(T, QH * 128, dtype=torch.float8_e4m3fn if fp8_out else torch.bfloat16, device=q.device)
    if fp8_out and out_scale is None:
        out_scale = torch.empty(sf_bytes(T, QH * 128), dtype=torch.uint8, device=q.device)
    if lse is not None and fp8_out:
        raise ValueError("a log-sum-exp output goes with a bf16 attention output")
    count_launch()
    native().prefill_attention_tc2(q, k_cache, v_cache, seqs, blocks, page_list, softmax_scale, out,
                                   out_scale if fp8_out else None, lse)
    return (out, out_scale) if fp8_out else out


def attention_merge(o_a, lse_a, o_b, lse_b, source, *, fp8_out: bool = True, out=None, out_scale=None):
    """Merge two attention reads of the same rows over disjoint key sets (csrc/attention_merge.cu).

    o_a bf16 [T, QH*D], lse_a fp32 [T, QH]: every row's read of one key set; o_b / lse_b
    [R, ...]: reads of another key set by some rows, `source` int32 [T] naming each row's
    row of o_b (-1: none). out = (o_a e^lse_a + o_b e^lse_b) / (e^lse_a + e^lse_b), as bf16
    or as e4m3 with UE8M0 scales per 32 columns in the MX atom layout (the next GEMM's input).
    """
    T, W = o_a.shape
    QH = lse_a.shape[1]
    if out is None:
        out = torch.empty(T, W, dtype=torch.float8_e4m3fn if fp8_out else torch.bfloat16, device=o_a.device)
    if fp8_out and out_scale is None:
        out_scale = torch.empty(sf_bytes(T, W), dtype=torch.uint8, device=o_a.device)
    count_launch()
    native().attention_merge(o_a, lse_a, o_b, lse_b, source, QH, out, out_scale if fp8_out else None)
    return (out, out_scale) if fp8_out else out


# (head_dim, q heads per KV head) pairs the small-tile attention kernel is built for
SMALL_ATTENTION_SHAPES = frozenset({(64, 1), (64, 2), (64, 4), (128, 1), (128, 4), (256, 2), (256, 4), (256, 6),
                                    (256, 8), (512, 8)})


def small_attention(q, k_cache, v_cache, seqs, tiles, dseqs, page_list, softmax_scale: float, out,
                    gate=None, gate_hstride: int = 0):
    """Small-tile paged attention (mma.sync) for head_dim 64 / 128 / 256, optional sigmoid gate.

    The shape is checked here, before the native call: only the (head_dim, group) pairs the
    kernel is instantiated for run.
    """
    D, G = q.shape[2], q.shape[1] // k_cache.shape[2]
    if (D, G) not in SMALL_ATTENTION_SHAPES:
        raise ValueError(f"small_attention: head_dim {D} with {G} q heads per KV head is not built; "
                         f"built: {sorted(SMALL_ATTENTION_SHAPES)}")
    count_launch(int(tiles.shape[0] > 0) + int(dseqs.numel() > 0))
    native().small_attention(q, k_cache, v_cache, seqs, tiles, dseqs, page_list, softmax_scale, out, gate,
                             gate_hstride)
    return out


def post_norm_add_norm(y: torch.Tensor, h: torch.Tensor, w_post: torch.Tensor, w_next=None, eps: float = 1e-5):
    """A sandwich-normed block's residual add: h += RMSNorm(y) * w_post in place; then, with
    w_next, the next block's input RMSNorm(h) * w_next (bf16 [T, H]), else None."""
    x = torch.empty_like(h) if w_next is not None else None
    count_launch()
    native().post_norm_add_norm(y, h, w_post, w_next, x, eps)
    return x


def kv_copy_rows(k_cache: torch.Tensor, v_cache: torch.Tensor, src: torch.Tensor, dst: torch.Tensor) -> None:
    """Copy the K and V rows of arena slots `src` to slots `dst` (int32, one per row)."""
    if src.numel():
        count_launch()
        native().kv_copy_rows(k_cache, v_cache, src, dst)


def chunk_attention(q, k_cache, v_cache, chunk, softmax_scale: float, *, mx: bool, tc: bool,
                    out=None, out_scale=None):
    """Attention of every query row of a packed chunk.

    Prefill tiles (sequences with several new tokens) run on the tcgen05
    kernel (`tc`, needs 4 q heads per KV head) or the mma.sync kernel; the
    chunk's one-token sequences run on the decode kernel. Both write their
    own rows of one output: e4m3 + MX scale atoms (`mx`) or bf16.
    """
    T, QH = q.shape[0], q.shape[1]
    if out is None:
        out = torch.empty(T, QH * 128, dtype=torch.float8_e4m3fn if mx else torch.bfloat16, device=q.device)
    if mx and out_scale is None:
        out_scale = torch.empty(sf_bytes(T, QH * 128), dtype=torch.uint8, device=q.device)
    tree = getattr(chunk, "tree", None)
    if tree is not None and tc and k_cache.shape[1] % 64 == 0 and chunk.tiles.shape[0] > 0:
        return _tree_attention(q, k_cache, v_cache, chunk, tree, softmax_scale, mx=mx, out=out, out_scale=out_scale)
    if chunk.tiles.shape[0] > 0:
        blocks = getattr(chunk, "blocks", None)
        if tc and blocks is not None and k_cache.shape[1] % 64 == 0:
            prefill_attention_tc2(q, k_cache, v_cache, chunk.seqs, blocks, chunk.page_list, softmax_scale,
                                  fp8_out=mx, out=out, out_scale=out_scale)
        elif tc:
            prefill_attention_tc(q, k_cache, v_cache, chunk.seqs, chunk.tiles, chunk.page_list, softmax_scale,
                                 fp8_out=mx, out=out, out_scale=out_scale)
        else:
            prefill_attention(q, k_cache, v_cache, chunk.seqs, chunk.tiles, chunk.page_list, softmax_scale,
                              fp8_out=mx, mx=mx, out=out, out_scale=out_scale)
    dseqs = getattr(chunk, "dseqs", None)
    if dseqs is not None and dseqs.numel() > 0:
        decode_attention(q, k_cache, v_cache, chunk.seqs, dseqs, chunk.page_list, softmax_scale, out,
                         out_scale if mx else None)
    return (out, out_scale) if mx else out


def _tree_attention(q, k_cache, v_cache, chunk, tree, softmax_scale, *, mx, out, out_scale):
    """The tree path of a chunk (engine/chunk.py): every row's own reads (persistent kernel,
    bf16 + log-sum-exp), the stacked readers' read of their shared segments (same kernel over
    the gathered rows), one-token rows on the decode kernel, then the merge (+ MX quantization)."""
    T, QH = q.shape[0], q.shape[1]
    o_a = torch.empty(T, QH * 128, dtype=torch.bfloat16, device=q.device)
    lse_a = torch.empty(T, QH, dtype=torch.float32, device=q.device)
    prefill_attention_tc2(q, k_cache, v_cache, tree["seqs_a"], tree["blocks_a"], chunk.page_list, softmax_scale,
                          fp8_out=False, out=o_a, lse=lse_a)
    dseqs = getattr(chunk, "dseqs", None)
    if dseqs is not None and dseqs.numel() > 0:
        decode_attention(q, k_cache, v_cache, chunk.seqs, dseqs, chunk.page_list, softmax_scale, o_a, None)
    rows = tree["rows"]
    qb = q.index_select(0, rows.long())
    o_b = torch.empty(rows.numel(), QH * 128, dtype=torch.bfloat16, device=q.device)
    lse_b = torch.empty(rows.numel(), QH, dtype=torch.float32, device=q.device)
    prefill_attention_tc2(qb, k_cache, v_cache, tree["seqs_b"], tree["blocks_b"], chunk.page_list, softmax_scale,
                          fp8_out=False, out=o_b, lse=lse_b)
    if mx:
        if out is None:
            out = torch.empty(T, QH * 128, dtype=torch.float8_e4m3fn, device=q.device)
        if out_scale is None:
            out_scale = torch.empty(sf_bytes(T, QH * 128), dtype=torch.uint8, device=q.device)
        attention_merge(o_a, lse_a, o_b, lse_b, tree["source"], fp8_out=True, out=out, out_scale=out_scale)
        return out, out_scale
    out = attention_merge(o_a, lse_a, o_b, lse_b, tree["source"], fp8_out=False, out=out)
    return out


def sae_features(x: torch.Tensor, w_enc: torch.Tensor, b_enc: torch.Tensor, keep: int) -> torch.Tensor:
    """SAE encode of residual rows x [R, H] bf16: [R, 2*keep] fp32 = keep feature ids, then strengths.

    The encode GEMM is the bf16 tcgen05 GEMM; csrc/sae.cu adds the bias and
    selects the `keep` largest per row (clamped at 0, strongest first).
    """
    pre = gemm(x.contiguous(), w_enc)
    out = torch.empty(x.shape[0], 2 * keep, dtype=torch.float32, device=x.device)
    count_launch()
    native().sae_topk(pre, b_enc, keep, out)
    return out


def final_norm_readout(x, rows, norm_w, eps: float, head_rows, *, logits=None, normed=None):
    """Gather rows of x, final RMSNorm, logits against the retained head rows."""
    _check_hidden(x.shape[1], "final_norm_readout")
    if logits is None:
        logits = torch.empty(rows.numel(), head_rows.shape[0], dtype=torch.float32, device=x.device)
    count_launch()
    native().final_norm_readout(x, rows, norm_w, eps, head_rows, logits, normed)
    return logits


def row_argmax_lse(logits: torch.Tensor):
    """Row-wise argmax and log-sum-exp of bf16 logits [R, V] -> (int32 [R], fp32 [R])."""
    R = logits.shape[0]
    arg = torch.empty(R, dtype=torch.int32, device=logits.device)
    lse = torch.empty(R, dtype=torch.float32, device=logits.device)
    count_launch()
    native().row_argmax_lse(logits, arg, lse)
    return arg, lse


READOUT_TOPK = 8   # candidates per row of a top-k readout (copy-constrained extraction)


def head_readout(normed: torch.Tensor, head: torch.Tensor, ans: torch.Tensor, topk: bool = False):
    """Full-vocabulary readout of final-normed rows: [answer logits | argmax | log-sum-exp],
    then with `topk` the READOUT_TOPK best token ids and their logits."""
    logits = gemm(normed, head)
    arg, lse = row_argmax_lse(logits)
    cols = [ans, arg.float()[:, None], lse[:, None]]
    if topk:
        v, i = torch.topk(logits, READOUT_TOPK, dim=1)
        cols += [i.float(), v.float()]
    return torch.cat(cols, dim=1)


def set_wait_budget(cycles: int, device: int = 0) -> None:
    """Spin budget, in clock cycles, of every bounded wait in the kernels on `device`
    (0 restores the default of about two seconds)."""
    native().set_wait_budget(device, int(cycles))


def read_and_clear_error(device: int = 0) -> int:
    """Synchronize and return (then clear) the kernels' bounded-wait error code."""
    return int(native().read_and_clear_error(device))
