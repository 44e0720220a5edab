"""Plain PyTorch fp32 statements of every kernel op.

These are the numerical oracle for the kernel tests and the ops of the CPU
model (`quail_b200.models.qwen3.Qwen3Reference`).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def rope_cos_sin(max_pos: int, head_dim: int, theta: float, device=None) -> torch.Tensor:
    """[max_pos, head_dim] fp32: cos of the head_dim/2 frequencies, then sin."""
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64, device=device) / half))
    pos = torch.arange(max_pos, dtype=torch.float64, device=device)
    ang = pos[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).float()


def rope_neox(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, D]: rotate (i, i + D/2) pairs by position."""
    D = x.shape[-1]
    half = D // 2
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def mrope_streams(pairs: int, sections) -> torch.Tensor:
    """[pairs] position stream (0 time, 1 height, 2 width) of each rotary frequency pair under
    interleaved multimodal RoPE: pair p follows height when p % 3 == 1 and p < 3 * sections[1],
    width when p % 3 == 2 and p < 3 * sections[2], else time."""
    p = torch.arange(pairs)
    s = torch.zeros(pairs, dtype=torch.long)
    s[(p % 3 == 1) & (p < 3 * sections[1])] = 1
    s[(p % 3 == 2) & (p < 3 * sections[2])] = 2
    return s


def rope_neox_3d(x: torch.Tensor, pos3: torch.Tensor, cos_sin: torch.Tensor, sections) -> torch.Tensor:
    """rope_neox with [T, 3] positions: each frequency pair rotates by its stream's position."""
    D = x.shape[-1]
    half = D // 2
    streams = mrope_streams(half, sections).to(pos3.device)
    rows = pos3.long()[:, streams]                               # [T, half] table row per pair
    cols = torch.arange(half, device=pos3.device)
    cos = cos_sin[rows, cols[None, :]][:, None, :]
    sin = cos_sin[rows, half + cols[None, :]][:, None, :]
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate.float()) * up.float()


def segmented_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        seqs: torch.Tensor, page_list: torch.Tensor, scale: float) -> torch.Tensor:
    """fp32 oracle of csrc/attention.cu: [T, QH, D] -> [T, QH * D].

    seqs[s, 3] holds flags: bit 0, the own segment is read both ways; bits 8..23, a
    sliding window over the own segment (0: none); bit 24, the window spans every segment
    (with bit 0 it bounds only the earlier segments).
    """
    T, QH, D = q.shape
    P, KH = k_cache.shape[1], k_cache.shape[2]
    out = torch.zeros(T, QH * D, dtype=torch.float32, device=q.device)
    seqs = seqs.cpu()
    pl = page_list.cpu()
    for s in range(seqs.shape[0]):
        q_start, q_len, nseg = (int(v) for v in seqs[s, :3])
        ks, vs, causal_from = [], [], 0
        for i in range(nseg):
            ln, off = int(seqs[s, 4 + i]), int(seqs[s, 8 + i])
            idx = torch.arange(ln)
            pages = pl[off + idx // P]
            slots = (pages * P + idx % P).to(k_cache.device)
            ks.append(k_cache.reshape(-1, KH, D)[slots].float())
            vs.append(v_cache.reshape(-1, KH, D)[slots].float())
            if i < nseg - 1:
                causal_from += ln
        k = torch.cat(ks)  # [L, KH, D]
        v = torch.cat(vs)
        L = k.shape[0]
        own_len = L - causal_from
        qs = q[q_start:q_start + q_len].float()  # [q_len, QH, D]
        rep = QH // KH
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
        scores = torch.einsum("qhd,khd->hqk", qs, k) * scale
        qpos = causal_from + own_len - q_len + torch.arange(q_len)
        kpos = torch.arange(L)
        mask = kpos[None, :] <= qpos[:, None]
        flags = int(seqs[s, 3])
        win = (flags >> 8) & 0xFFFF
        win_all = bool(flags & (1 << 24))
        if flags & 1:                 # own segment read both ways (document-isolated block, canvas)
            mask = torch.ones_like(mask)
            if win and win_all:
                mask &= (kpos[None, :] >= causal_from) | (kpos[None, :] > qpos[:, None] - win)
        elif win and win_all:         # a sliding window over the whole sequence
            mask &= kpos[None, :] > qpos[:, None] - win
        elif win:                     # a sliding window over the own segment; earlier segments whole
            mask &= (kpos[None, :] < causal_from) | (kpos[None, :] > qpos[:, None] - win)
        scores = scores.masked_fill(~mask.to(scores.device)[None], float("-inf"))
        p = torch.softmax(scores, dim=-1)
        o = torch.einsum("hqk,khd->qhd", p, v)
        out[q_start:q_start + q_len] = o.reshape(q_len, QH * D)
    return out


def segmented_attention_lse(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            seqs: torch.Tensor, page_list: torch.Tensor, scale: float):
    """segmented_attention plus each covered row's log-sum-exp: ([T, QH * D], [T, QH]);
    rows no sequence covers get out 0 and lse -inf."""
    T, QH, D = q.shape
    P, KH = k_cache.shape[1], k_cache.shape[2]
    out = torch.zeros(T, QH * D, dtype=torch.float32, device=q.device)
    lse = torch.full((T, QH), float("-inf"), dtype=torch.float32, device=q.device)
    seqs = seqs.cpu()
    pl = page_list.cpu()
    for s in range(seqs.shape[0]):
        q_start, q_len, nseg = (int(v) for v in seqs[s, :3])
        ks, vs, before = [], [], 0
        for i in range(nseg):
            ln, off = int(seqs[s, 4 + i]), int(seqs[s, 8 + i])
            idx = torch.arange(ln)
            slots = (pl[off + idx // P] * P + idx % P).to(k_cache.device)
            ks.append(k_cache.reshape(-1, KH, D)[slots].float())
            vs.append(v_cache.reshape(-1, KH, D)[slots].float())
            if i < nseg - 1:
                before += ln
        k, v = torch.cat(ks), torch.cat(vs)
        L = k.shape[0]
        qs = q[q_start:q_start + q_len].float()
        k = k.repeat_interleave(QH // KH, dim=1)
        v = v.repeat_interleave(QH // KH, dim=1)
        sc = torch.einsum("qhd,khd->hqk", qs, k) * scale
        qpos = L - q_len + torch.arange(q_len)
        kpos = torch.arange(L)
        mask = kpos[None, :] <= qpos[:, None]
        if int(seqs[s, 3]) & 1:
            mask = torch.ones_like(mask)
        sc = sc.masked_fill(~mask.to(sc.device)[None], float("-inf"))
        l_ = torch.logsumexp(sc, dim=-1)                       # [QH, q_len]
        p = torch.exp(sc - l_[..., None]).nan_to_num(0.0)
        out[q_start:q_start + q_len] = torch.einsum("hqk,khd->qhd", p, v).reshape(q_len, QH * D)
        lse[q_start:q_start + q_len] = l_.t()
    return out, lse


def merge_lse(o_a: torch.Tensor, lse_a: torch.Tensor, o_b: torch.Tensor, lse_b: torch.Tensor,
              source: torch.Tensor) -> torch.Tensor:
    """fp32 statement of csrc/attention_merge.cu: rows with source >= 0 merge o_a with o_b[source]
    by their log-sum-exps; the others keep o_a."""
    T, W = o_a.shape
    QH = lse_a.shape[1]
    D = W // QH
    out = o_a.float().clone().view(T, QH, D)
    rows = (source >= 0).nonzero().flatten()
    if rows.numel():
        src = source[rows].long()
        la, lb = lse_a[rows].float(), lse_b[src].float()
        m = torch.maximum(la, lb)
        wa, wb = torch.exp(la - m).nan_to_num(0.0), torch.exp(lb - m).nan_to_num(0.0)
        z = (wa + wb).clamp(min=1e-30)
        a = o_a.float().view(T, QH, D)[rows]
        b = o_b.float().view(-1, QH, D)[src]
        out[rows] = (a * wa[..., None] + b * wb[..., None]) / z[..., None]
    return out.view(T, W)


def tree_attention(q, k_cache, v_cache, seqs, page_list, tree: dict, scale: float) -> torch.Tensor:
    """The tree path in fp32: each row's read without the stacked shared segment (seqs_a), the
    stacked readers' read of the shared segments (seqs_b over rows q[rows]), merged."""
    o_a, lse_a = segmented_attention_lse(q, k_cache, v_cache, tree["seqs_a"], page_list, scale)
    qb = q[tree["rows"].long()]
    o_b, lse_b = segmented_attention_lse(qb, k_cache, v_cache, tree["seqs_b"], page_list, scale)
    # rows the tree tables do not cover (one-token sequences) read as in the unified path
    uncovered = torch.isinf(lse_a).all(dim=1) & (tree["source"].cpu() < 0).to(lse_a.device)
    if bool(uncovered.any()):
        full = segmented_attention(q, k_cache, v_cache, seqs, page_list, scale)
        o_a[uncovered] = full[uncovered]
    return merge_lse(o_a, lse_a, o_b, lse_b, tree["source"].to(o_a.device))


def attention_tiles(seqs: torch.Tensor, block_q: int = 32) -> torch.Tensor:
    """[n_tiles, 2] int32 (sequence, first query row) covering every query row."""
    rows = []
    for s in range(seqs.shape[0]):
        q_len = int(seqs[s, 1])
        for q0 in range(0, q_len, block_q):
            rows.append((s, q0))
    if not rows:
        return torch.zeros(0, 2, dtype=torch.int32)
    return torch.tensor(rows, dtype=torch.int32)


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


def moe_route(logits: torch.Tensor, top_k: int):
    """Qwen3-MoE routing: softmax over experts (fp32), top-k, weights renormalized to sum 1.

    Returns (expert ids [T, k] int64, weights [T, k] fp32).
    """
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = p.topk(top_k, dim=-1)
    return ids, w / w.sum(dim=-1, keepdim=True)


def sae_features(x: torch.Tensor, w_enc: torch.Tensor, b_enc: torch.Tensor, keep: int) -> torch.Tensor:
    """fp32 statement of the SAE readout: [R, 2*keep] = top-keep feature ids, then strengths (>= 0)."""
    pre = x.float() @ w_enc.float().t() + b_enc.float()
    v, i = pre.topk(keep, dim=1)
    v = v.clamp(min=0.0)
    i = torch.where(v > 0, i, torch.zeros_like(i))
    return torch.cat([i.float(), v], dim=1)


def head_readout(full: torch.Tensor, ans: torch.Tensor, topk: bool = False, k: int = 8) -> torch.Tensor:
    """fp32 statement of ops.head_readout from full-vocabulary logits [R, V]."""
    cols = [ans, full.argmax(dim=1).float()[:, None], torch.logsumexp(full, dim=1)[:, None]]
    if topk:
        v, i = torch.topk(full, k, dim=1)
        cols += [i.float(), v.float()]
    return torch.cat(cols, dim=1)
