"""LFM3 (LiquidAI d1) under set attention: whole-sequence passes, no KV kept.

Each layer is sandwich-normed:

    x = RMSNorm(h) * operator_norm;  y = mixer(x);  h += RMSNorm(y) * post_operator_norm
    x = RMSNorm(h) * ffn_norm;       y = SwiGLU(x);  h += RMSNorm(y) * post_ffn_norm

Mixers:
  conv  B, C, x = in_proj(x);  y = out_proj(C * causal_depthwise_conv(B * x)), 7 taps, from a
        zero window at the start of every pass.
  attn  full attention: q, k, v and one gate logit per head from one projection; per-head
        RMSNorm of q and k; NeoX rotary over the first `rotary_pairs` share of the frequency
        pairs (the rest unrotated); the output of each head times sigmoid(gate); o_proj.
        Under set attention the state rows (prompt head, document, state tail) read the whole
        pass both ways and each question reads the state and itself, both ways.
  swa   the same projection with full rotary, causal over the pass with a sliding window.

A pass (`SetPass`) is a state and up to `set_size` questions; `forward_passes` returns the
final-normed hidden rows each pass asks for. `Lfm3Reference` is the fp32 statement (dense
masks, CPU or GPU); `Lfm3Pipeline` runs the sm_100a kernels: each pass's keys go to pages
of a scratch arena, the state rows read the pass as one bidirectional sequence, and every
question's keys are also copied to its own pages, so a question is a two-segment
sequence (the state, then itself, read both ways) on the same attention kernel; the
sliding layers read the pass as one causal sequence with a window.

Reference: quail/backends/quail/executor/models/lfm3.py:113-463 (Lfm3Pipeline, the
set-attention reads merged by log-sum-exp) and lfm3_kernels.py (gated conv, sandwich norm,
head gates); HF names of LFM3 checkpoints (model.layers.N.{operator_norm, conv.*, self_attn.*,
feed_forward.*}).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from quail_b200.models.config import DecoderConfig
from quail_b200.models.weights import dequantized, final_norm_name
from quail_b200.ops import reference as ref


@dataclass
class SetPass:
    """One set-attention pass: `tokens` = the state, then each question's tokens."""

    tokens: np.ndarray
    state: int                          # rows of the state (prompt head, document, state tail)
    questions: list = field(default_factory=list)   # each question's length, in order
    read_rows: list = field(default_factory=list)   # pass rows whose final-normed hidden state is returned

    @property
    def length(self) -> int:
        return len(self.tokens)


def rotary_table(cfg: DecoderConfig, kind: str, device=None) -> torch.Tensor:
    """[max_position, D] fp32 cos | sin. Full-attention layers keep the whole head's frequency
    progression and zero the frequencies past `rotary_pairs` (those pairs stay unrotated);
    the table is rounded to bf16 as the checkpoints' own code rounds it."""
    t = ref.rope_cos_sin(cfg.max_position, cfg.head_dim, cfg.rope_theta, device=device)
    half = cfg.head_dim // 2
    if kind == "attn" and cfg.rotary_pairs < 1.0:
        keep = int(cfg.rotary_pairs * half)
        t[:, keep:half] = 1.0
        t[:, half + keep:] = 0.0
    return t.bfloat16().float()


def set_mask(p: SetPass, kind: str, window: int) -> torch.Tensor:
    """[L, L] bool: which keys each row of the pass reads in a layer of `kind`."""
    L = p.length
    i = torch.arange(L)[:, None]
    j = torch.arange(L)[None, :]
    if kind == "swa":
        return (j <= i) & (j > i - window)
    mask = torch.zeros(L, L, dtype=torch.bool)
    mask[:p.state, :] = True                     # the state reads the whole pass
    start = p.state
    for n in p.questions:
        mask[start:start + n, :p.state] = True   # a question reads the state ...
        mask[start:start + n, start:start + n] = True   # ... and itself, both ways
        start += n
    return mask


class Lfm3Reference:
    """fp32 forward of set-attention passes (dense per-pass masks)."""

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor], device="cpu", dtype=torch.float32):
        assert cfg.arch == "lfm3"
        self.cfg = cfg
        self.device = device
        f = lambda t: t.to(device=device, dtype=dtype)  # noqa: E731
        self.embed = f(ckpt["model.embed_tokens.weight"])
        self.final_norm = f(ckpt[final_norm_name(cfg)])
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            L = {n: f(ckpt[p + n + ".weight"]) for n in ("operator_norm", "post_operator_norm", "ffn_norm",
                                                          "post_ffn_norm")}
            L.update(w1=f(dequantized(ckpt, p + "feed_forward.w1")), w3=f(dequantized(ckpt, p + "feed_forward.w3")),
                     w2=f(dequantized(ckpt, p + "feed_forward.w2")))
            if cfg.kind(i) == "conv":
                L.update(win=f(dequantized(ckpt, p + "conv.in_proj")), wout=f(dequantized(ckpt, p + "conv.out_proj")),
                         taps=f(ckpt[p + "conv.conv.weight"][:, 0, :]))
            else:
                a = p + "self_attn."
                L.update(wq=f(dequantized(ckpt, a + "q_proj")), wk=f(dequantized(ckpt, a + "k_proj")),
                         wv=f(dequantized(ckpt, a + "v_proj")), wg=f(dequantized(ckpt, a + "gate_proj")),
                         wo=f(dequantized(ckpt, a + "o_proj")), qn=f(ckpt[a + "q_norm.weight"]),
                         kn=f(ckpt[a + "k_norm.weight"]))
            self.layers.append(L)
        self.head = f(self.embed if cfg.tied_head else ckpt["lm_head.weight"])
        self.tables = {k: rotary_table(cfg, k, device) for k in ("attn", "swa")}
        self.scale = ref.softmax_scale(cfg.head_dim)

    def _norm(self, x, w):
        return ref.rmsnorm(x, w, self.cfg.rms_eps)

    def _conv(self, L, x):
        H, W = self.cfg.hidden, self.cfg.conv_width
        bcx = x @ L["win"].t()
        B, C, xx = bcx[:, :H], bcx[:, H:2 * H], bcx[:, 2 * H:]
        bx = torch.cat([torch.zeros(W - 1, H, dtype=x.dtype, device=x.device), B * xx])
        n = x.shape[0]
        acc = torch.zeros(n, H, dtype=x.dtype, device=x.device)
        for j in range(W):
            acc += bx[j:j + n] * L["taps"][:, j]
        return (C * acc) @ L["wout"].t()

    def _attention(self, L, x, p: SetPass, kind: str):
        cfg = self.cfg
        QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        n = x.shape[0]
        pos = torch.arange(n, device=x.device)
        q = ref.rope_neox(self._norm((x @ L["wq"].t()).view(n, QH, D), L["qn"]), pos, self.tables[kind])
        k = ref.rope_neox(self._norm((x @ L["wk"].t()).view(n, KH, D), L["kn"]), pos, self.tables[kind])
        v = (x @ L["wv"].t()).view(n, KH, D)
        g = x @ L["wg"].t()                                   # [n, QH] one gate logit per head
        rep = QH // KH
        k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
        s = torch.einsum("qhd,khd->hqk", q, k) * self.scale
        s = s.masked_fill(~set_mask(p, kind, cfg.sliding_window).to(x.device)[None], float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), v)
        o = o * torch.sigmoid(g)[:, :, None]
        return o.reshape(n, QH * D) @ L["wo"].t()

    @torch.no_grad()
    def forward_passes(self, passes: list[SetPass]) -> list[torch.Tensor]:
        cfg = self.cfg
        out = []
        for p in passes:
            h = self.embed[torch.as_tensor(p.tokens, dtype=torch.long, device=self.device)]
            for i, L in enumerate(self.layers):
                x = self._norm(h, L["operator_norm"])
                kind = cfg.kind(i)
                y = self._conv(L, x) if kind == "conv" else self._attention(L, x, p, kind)
                h = h + self._norm(y, L["post_operator_norm"])
                x = self._norm(h, L["ffn_norm"])
                y = ref.silu_mul(x @ L["w1"].t(), x @ L["w3"].t()) @ L["w2"].t()
                h = h + self._norm(y, L["post_ffn_norm"])
            rows = torch.as_tensor(list(p.read_rows), dtype=torch.long, device=self.device)
            out.append(self._norm(h[rows], self.final_norm).float())
        return out


class Lfm3Pipeline:
    """Set-attention passes of an LFM3 model on the GPU kernels (bf16 weights)."""

    PAGE = 16            # scratch-arena page: question keys are short

    def __init__(self, cfg: DecoderConfig, ckpt: dict[str, torch.Tensor], device, max_tokens: int = 16384):
        from quail_b200.ops.quant import interleave_gate_up
        assert cfg.arch == "lfm3" and cfg.head_dim in (64, 128, 256)
        self.cfg = cfg
        self.device = torch.device(device)
        bf = torch.bfloat16
        H, QH, KH, D = cfg.hidden, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim

        def proj(name):
            return dequantized(ckpt, name).to(device=device, dtype=bf).contiguous()

        def vec(name):
            return ckpt[name].to(device=device, dtype=bf).contiguous()

        self.embed = ckpt["model.embed_tokens.weight"].to(device=device, dtype=bf).contiguous()
        self.final_norm = vec(final_norm_name(cfg))
        # q | k | v | per-head gate logits, the gate rows padded to a 128-row block
        self.gate_col = QH * D + 2 * KH * D
        pad = -(-QH // 128) * 128 - QH
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            L = {n: vec(p + n + ".weight") for n in ("operator_norm", "post_operator_norm", "ffn_norm",
                                                      "post_ffn_norm")}
            L["wgu"] = interleave_gate_up(torch.cat([proj(p + "feed_forward.w1"), proj(p + "feed_forward.w3")]))
            L["wd"] = proj(p + "feed_forward.w2")
            if cfg.kind(i) == "conv":
                L.update(win=proj(p + "conv.in_proj"), wout=proj(p + "conv.out_proj"),
                         taps=ckpt[p + "conv.conv.weight"][:, 0, :].to(device=device, dtype=torch.float32)
                         .contiguous())
            else:
                a = p + "self_attn."
                parts = [proj(a + "q_proj"), proj(a + "k_proj"), proj(a + "v_proj"), proj(a + "gate_proj")]
                if pad:
                    parts.append(torch.zeros(pad, H, dtype=bf, device=device))
                L.update(wqkvg=torch.cat(parts).contiguous(), wo=proj(a + "o_proj"), qn=vec(a + "q_norm.weight"),
                         kn=vec(a + "k_norm.weight"))
            self.layers.append(L)
        self.head = (self.embed if cfg.tied_head else ckpt["lm_head.weight"].to(device=device, dtype=bf))
        self.tables = {k: rotary_table(cfg, k, device).contiguous() for k in ("attn", "swa")}
        self.scale = ref.softmax_scale(D)
        self.max_tokens = max_tokens
        # scratch KV pages: every pass's rows, plus each question's own copy
        pages = 2 * (max_tokens // self.PAGE) + 1024
        n_attn = len(cfg.attn_layers)
        self.kc = torch.empty(n_attn, pages, self.PAGE, KH, D, dtype=bf, device=device)
        self.vc = torch.empty_like(self.kc)
        self.num_pages = pages
        self.conv_state = torch.zeros(1, 1, cfg.conv_width - 1, H, dtype=torch.float32, device=device)

    def _layout(self, passes: list[SetPass]):
        """Host-side metadata of a chunk of passes: ids, positions, KV slots, the question-key
        copies, and the sequence tables of the full and sliding layers."""
        P = self.PAGE
        ids, pos, slots, src, dst = [], [], [], [], []
        full, swa, convs, reads = [], [], [], []
        row0 = page = 0
        win = self.cfg.sliding_window
        for p in passes:
            L = p.length
            ids.append(np.asarray(p.tokens, dtype=np.int32))
            pos.append(np.arange(L, dtype=np.int32))
            base = page
            page += -(-L // P)
            slots.append(base * P + np.arange(L, dtype=np.int32))
            # the state reads the whole pass both ways; the sliding layers read it causally
            full.append([row0, p.state, 1, 1, L, 0, 0, 0, base, 0, 0, 0])
            swa.append([row0, L, 1, win << 8, L, 0, 0, 0, base, 0, 0, 0])
            convs.append([row0, L] + [0] * 10)
            start = p.state
            for n in p.questions:
                qbase = page
                page += -(-n // P)
                src.append(base * P + start + np.arange(n, dtype=np.int32))
                dst.append(qbase * P + np.arange(n, dtype=np.int32))
                full.append([row0 + start, n, 2, 1, p.state, n, 0, 0, base, qbase, 0, 0])
                start += n
            reads.append(row0 + np.asarray(p.read_rows, dtype=np.int64))
            row0 += L
        if page > self.num_pages:
            raise ValueError(f"the passes need {page} scratch pages; the pipeline has {self.num_pages}")

        def cat(parts, dtype):
            return np.concatenate(parts).astype(dtype) if parts else np.zeros(0, dtype)
        return (cat(ids, np.int32), cat(pos, np.int32), cat(slots, np.int32), cat(src, np.int32), cat(dst, np.int32),
                np.asarray(full, np.int32).reshape(-1, 12), np.asarray(swa, np.int32).reshape(-1, 12),
                np.asarray(convs, np.int32).reshape(-1, 12), reads, page)

    @torch.no_grad()
    def forward_passes(self, passes: list[SetPass]) -> list[torch.Tensor]:
        from quail_b200 import ops
        cfg = self.cfg
        dev = self.device
        QH, KH, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        ids, pos, slots, src, dst, full, swa, convs, reads, pages = self._layout(passes)
        T = len(ids)
        if T == 0:
            return []

        def up(a):
            return torch.from_numpy(a).to(dev, non_blocking=True)
        ids_d, pos_d, slots_d, src_d, dst_d = up(ids), up(pos), up(slots), up(src), up(dst)
        full_d, swa_d, conv_d = up(full), up(swa), up(convs)
        page_list = torch.arange(pages, dtype=torch.int32, device=dev)
        tiles = {"attn": ref.attention_tiles(torch.from_numpy(full)).to(dev),
                 "swa": ref.attention_tiles(torch.from_numpy(swa)).to(dev)}
        seqs = {"attn": full_d, "swa": swa_d}
        no_decode = torch.zeros(0, dtype=torch.int32, device=dev)
        sio = torch.full((len(passes), 2), -1, dtype=torch.int32, device=dev)
        C = ops.native()
        h = ops.embed_gather(ids_d, self.embed)
        x = ops.rmsnorm_quant(h, self.layers[0]["operator_norm"], cfg.rms_eps, fp8=False)
        ai = 0
        for i, L in enumerate(self.layers):
            kind = cfg.kind(i)
            if kind == "conv":
                bcx = ops.gemm(x, L["win"])
                yc = torch.empty(T, cfg.hidden, dtype=torch.bfloat16, device=dev)
                ops.count_launch()
                C.short_conv(bcx, L["taps"], conv_d, sio, self.conv_state, 0, yc)
                y = ops.gemm(yc, L["wout"])
            else:
                p = ops.gemm(x, L["wqkvg"])
                kc, vc = self.kc[ai], self.vc[ai]
                q = torch.empty(T, QH, D, dtype=torch.bfloat16, device=dev)
                ops.count_launch()
                C.hybrid_qk_rope_kv(p, QH, KH, False, pos_d, L["qn"], L["kn"], False, self.tables[kind], slots_d,
                                    kc, vc, q, cfg.rms_eps, 0, 0)
                if kind == "attn":
                    ops.kv_copy_rows(kc, vc, src_d, dst_d)
                o = torch.empty(T, QH * D, dtype=torch.bfloat16, device=dev)
                ops.small_attention(q, kc, vc, seqs[kind], tiles[kind], no_decode, page_list, self.scale, o,
                                    p[:, self.gate_col:], -1)
                y = ops.gemm(o, L["wo"])
                ai += 1
            x = ops.post_norm_add_norm(y, h, L["post_operator_norm"], L["ffn_norm"], cfg.rms_eps)
            a = ops.gemm(x, L["wgu"], epi=ops.EPI_SWIGLU_BF16)
            y = ops.gemm(a, L["wd"])
            nxt = self.layers[i + 1]["operator_norm"] if i + 1 < cfg.layers else None
            x = ops.post_norm_add_norm(y, h, L["post_ffn_norm"], nxt, cfg.rms_eps)
        counts = [len(r) for r in reads]
        rows = torch.from_numpy(np.concatenate(reads).astype(np.int32)).to(dev)
        normed = torch.empty(rows.numel(), cfg.hidden, dtype=torch.bfloat16, device=dev)
        # the final norm of the read rows (the readout's logits against one dummy head row are unused)
        ops.final_norm_readout(h, rows, self.final_norm, cfg.rms_eps, self.head[:8].contiguous(), normed=normed)
        return list(normed.float().split(counts))
