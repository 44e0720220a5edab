"""Packed prefill chunks: many questions' new tokens in one forward pass.

A chunk is the unit the GPU runs: up to `chunk_tokens` new tokens from many
sequences, plus the metadata the kernels read:

  ids, positions, slots   [T] int32  token id, absolute position, KV slot (page*P + offset; -1 = none)
  seqs                    [S, 12]    q_start, q_len, nseg, flags (bit 0: own segment both ways),
                                     seg_len[4], seg_off[4]
  tiles                   [n, 2]     (sequence, first query token) per 32-token prefill-attention tile
  blocks                  [m, 2]     the same per 64-token block of the persistent attention kernel,
                                     the blocks reading the most keys first
  dseqs                   [d]        sequences with one new token (decode attention: one CTA per KV head)
  state_io                [S, 2]     hybrid models: state slot each sequence starts from (-1 = zeros), slot it ends in
  page_list               [*]        page ids of every segment, segments point into it
  final_rows              [R]        token row whose logits each readout reads

The host packs it with numpy into one pinned int32 buffer and ships it with
a single H2D copy (reference: chunk.py pack_chunk + InputStaging, which
stage per-field pinned buffers).

The tree path (`ChunkPacker(tree=...)`): when several prefill sequences of a
chunk read the same resident segment first (the shared instruction prefix, a
join anchor), `Chunk.tree` also holds
  seqs_a   [S, 12]  the sequences without that stacked segment (every row's own reads)
  seqs_b   [G, 12]  one sequence per stacked segment: its readers' rows, stacked, read it whole
  blocks_a / blocks_b  the persistent attention kernel's blocks of each table
  rows     [R]      the chunk rows stacked into seqs_b's query rows, in order
  source   [T]      each chunk row's stacked row, -1 for none
and the attention runs as two reads merged by their log-sum-exps
(ops.attention_merge); `chunk.seqs` stays the unified table.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

MAX_SEGMENTS = 4
SEQ_INTS = 12
# the metadata arrays in upload order
PARTS = ("ids", "positions", "slots", "seqs", "tiles", "page_list", "final_rows", "dseqs", "state_io",
         "blocks")
ATTN_BLOCK_Q = 32


@dataclass
class SeqSpec:
    """One sequence of a chunk."""

    reads: list            # [(key, tokens)] earlier segments read in full (shared prefix, document, ...)
    own_key: object        # key whose pages receive the new tokens
    own_start: int         # own tokens already resident before this chunk
    tokens: np.ndarray     # new token ids
    pos_start: int         # absolute position of tokens[0]
    readout: bool = False  # read the logits of the last new token
    tag: object = None
    readout_rows: tuple | None = None  # offsets of new tokens to read (default: the last one)
    full: bool = False     # also read argmax and log-sum-exp over the whole vocabulary
    topk: bool = False     # and the best few token ids with their logits
    bidirectional: bool = False  # every own token reads every own token (a document-isolated block)


@dataclass
class Chunk:
    num_tokens: int
    ids: torch.Tensor
    positions: torch.Tensor
    slots: torch.Tensor
    seqs: torch.Tensor
    tiles: torch.Tensor
    page_list: torch.Tensor
    final_rows: torch.Tensor
    readout_tags: list = field(default_factory=list)
    dseqs: torch.Tensor | None = None
    state_io: torch.Tensor | None = None
    blocks: torch.Tensor | None = None
    num_seqs: int = 0
    host: dict | None = None   # numpy copies (tests, CPU reference)
    upload_bytes: int = 0
    full_readout: bool = False  # readout rows also need full-vocabulary argmax / log-sum-exp
    topk: bool = False          # and the top-k token ids and logits (ops.READOUT_TOPK)
    tree: dict | None = None    # the tree path's tables (module docstring), None: unified
    rope3: torch.Tensor | None = None   # [T, 3] rotary (time, height, width) positions of a model with images


TREE_BLOCK = 64        # query rows per block of the persistent attention kernel


def tree_saves(reader_rows: list, shared_tokens: int) -> bool:
    """The tree path's cost rule (the reference's cheaper_attention_path, cost/budgets.rs:537-562,
    restated for this kernel): the unified path reads the shared keys once per 64-row block of
    every reader, the tree path once per 64-row block of the stacked readers plus a merge pass;
    stack when that saves at least a quarter of the shared-key tiles and 16 tiles."""
    kv_tiles = -(-shared_tokens // TREE_BLOCK)
    unified = sum(-(-n // TREE_BLOCK) for n in reader_rows) * kv_tiles
    stacked = -(-sum(reader_rows) // TREE_BLOCK) * kv_tiles
    return unified - stacked >= max(16, unified // 4)


class ChunkPacker:
    """Packs SeqSpecs against a PagePool into a Chunk on `device`.

    tree: "unified" (never stack), "tree" (stack every shared first segment read by two or
    more prefill sequences) or "auto" (stack where `tree_saves` says so)."""

    def __init__(self, pool, device, pin: bool = True, split_decode: bool = True, tree: str = "unified",
                 tree_min_tokens: int = 64):
        if tree not in ("unified", "tree", "auto"):
            raise ValueError(f"attention path is 'unified', 'tree' or 'auto', not {tree!r}")
        # a model with a vision tower: the engine's ImageStore; each chunk then carries the
        # multimodal rotary positions of its tokens, and `rope_shift` what each key's image
        # tokens moved its rotary positions behind its KV positions
        self.images = None
        self.rope_shift: dict = {}
        self.tree = tree
        self.tree_min_tokens = tree_min_tokens
        self.pool = pool
        # one-token sequences go to the decode attention kernel instead of prefill tiles
        self.split_decode = split_decode
        self.device = torch.device(device)
        self.pin = pin and self.device.type == "cuda"
        self._staging: torch.Tensor | None = None

    def pack(self, specs: list[SeqSpec]) -> Chunk:
        host, tags = self.host_parts(specs)
        n_tok = host["ids"].size
        parts = [host[k] for k in PARTS]
        sizes = [p.size for p in parts]
        flat = np.concatenate([p.reshape(-1) for p in parts]) if n_tok else np.zeros(0, dtype=np.int32)
        dev = self._upload(flat)
        views = []
        o = 0
        for sz in sizes:
            views.append(dev[o:o + sz])
            o += sz
        rope3 = None
        if self.images is not None and n_tok:
            r3 = self.rope3_parts(specs)
            host["rope3"] = r3
            rope3 = self._upload_plain(r3.reshape(-1)).view(-1, 3)
        tree = self.tree_parts(specs, host) if self.tree != "unified" and n_tok else None
        tree_dev = None
        up = int(flat.nbytes)
        if tree is not None:
            keys = ("seqs_a", "seqs_b", "blocks_a", "blocks_b", "rows", "source")
            tflat = np.concatenate([tree[k].reshape(-1) for k in keys])
            tdev = self._upload_plain(tflat)
            tree_dev, o = {}, 0
            for k in keys:
                n = tree[k].size
                v = tdev[o:o + n]
                tree_dev[k] = v.view(-1, SEQ_INTS) if k.startswith("seqs") else (
                    v.view(-1, 2) if k.startswith("blocks") else v)
                o += n
            up += int(tflat.nbytes)
            host["tree"] = tree
        return Chunk(num_tokens=n_tok, ids=views[0], positions=views[1], slots=views[2],
                     seqs=views[3].view(-1, SEQ_INTS), tiles=views[4].view(-1, 2), page_list=views[5],
                     final_rows=views[6], dseqs=views[7], state_io=views[8].view(-1, 2),
                     blocks=views[9].view(-1, 2), readout_tags=tags, tree=tree_dev, rope3=rope3,
                     num_seqs=len(specs), host=host, upload_bytes=up,
                     full_readout=any(s.full and s.readout for s in specs),
                     topk=any(s.topk and s.readout for s in specs))

    def host_parts(self, specs: list[SeqSpec]) -> tuple[dict, list]:
        """The chunk's metadata as numpy arrays (keys of PARTS) and its readout tags.

        Built in Python lists and converted once: a decode pass has a thousand
        one-token sequences, so per-sequence numpy calls would dominate."""
        P = self.pool.page_tokens
        owned = self.pool.owned
        ids: list[int] = []
        pos: list[int] = []
        slots: list[int] = []
        seqs: list[int] = []
        state_io: list[int] = []
        slots_on = self.pool.state_slots > 0
        slot_of = self.pool.slot_of if slots_on else None
        page_list: list[int] = []
        seg_cache: dict = {}
        tiles: list[int] = []
        blocks: list[tuple] = []      # (keys read, sequence, first token)
        dseqs: list[int] = []
        final_rows: list[int] = []
        tags: list = []
        split = self.split_decode
        q = 0
        for si, s in enumerate(specs):
            toks = s.tokens
            n = len(toks)
            reads = s.reads
            nr = len(reads)
            if nr + 1 > MAX_SEGMENTS:
                raise ValueError(f"a sequence reads at most {MAX_SEGMENTS - 1} earlier segments")
            own = owned[s.own_key]
            j0 = s.own_start
            if n == 1:
                ids.append(int(toks[0]))
                pos.append(s.pos_start)
                slots.append(own[j0 // P] * P + j0 % P)
            else:
                ids.extend(toks.tolist() if hasattr(toks, "tolist") else toks)
                pos.extend(range(s.pos_start, s.pos_start + n))
                slots.extend(own[j // P] * P + j % P for j in range(j0, j0 + n))
            # int 3: flags; bit 0 = the own segment is read both ways (no causal mask)
            row = [q, n, nr + 1, 1 if s.bidirectional else 0, 0, 0, 0, 0, 0, 0, 0, 0]
            if slots_on:
                # continue the key's own state, else start from the last segment it reads
                dst = slot_of[s.own_key]
                src = dst if j0 > 0 else (slot_of[reads[-1][0]] if reads else -1)
                state_io += (src, dst)
            for i, (key, ln) in enumerate(reads):
                npg = -(-ln // P)
                ck = (key, npg)
                off = seg_cache.get(ck)
                if off is None:
                    off = len(page_list)
                    page_list.extend(owned[key][:npg])
                    seg_cache[ck] = off
                row[4 + i] = ln
                row[8 + i] = off
            own_len = j0 + n
            row[4 + nr] = own_len
            row[8 + nr] = len(page_list)
            page_list.extend(own[:-(-own_len // P)])
            seqs += row
            if n == 1 and split:
                dseqs.append(si)
            else:
                for q0 in range(0, n, ATTN_BLOCK_Q):
                    tiles += (si, q0)
                before = sum(ln for _, ln in reads)
                for q0 in range(0, n, 2 * ATTN_BLOCK_Q):
                    blocks.append((before + j0 + min(n, q0 + 2 * ATTN_BLOCK_Q), si, q0))
            if s.readout:
                if s.readout_rows is None:
                    final_rows.append(q + n - 1)
                else:
                    final_rows.extend(q + o for o in s.readout_rows)
                tags.append(s.tag)
            q += n
        i32 = np.int32
        S = len(specs)
        sio = np.asarray(state_io, dtype=i32).reshape(S, 2) if slots_on else np.full((S, 2), -1, dtype=i32)
        host = {"ids": np.asarray(ids, dtype=i32), "positions": np.asarray(pos, dtype=i32),
                "slots": np.asarray(slots, dtype=i32), "seqs": np.asarray(seqs, dtype=i32).reshape(S, SEQ_INTS),
                "tiles": np.asarray(tiles, dtype=i32).reshape(-1, 2), "page_list": np.asarray(page_list, dtype=i32),
                "final_rows": np.asarray(final_rows, dtype=i32), "dseqs": np.asarray(dseqs, dtype=i32),
                "state_io": sio,
                "blocks": np.asarray([(b[1], b[2]) for b in sorted(blocks, key=lambda b: -b[0])],
                                     dtype=i32).reshape(-1, 2)}
        return host, tags

    def rope3_parts(self, specs: list[SeqSpec]) -> np.ndarray:
        """[T, 3] int32 rotary positions of the chunk's tokens (engine/images.py)."""
        parts = []
        for s in specs:
            shift = sum(self.rope_shift.get(k, 0) for k, _ in s.reads)
            if s.own_start > 0:
                shift = self.rope_shift.get(s.own_key, shift)
            n = len(s.tokens)
            r3, shift = self.images.rope_positions(s.tokens, np.arange(s.pos_start, s.pos_start + n), shift)
            self.rope_shift[s.own_key] = shift
            parts.append(r3)
        return np.concatenate(parts).astype(np.int32)

    def tree_parts(self, specs: list[SeqSpec], host: dict) -> dict | None:
        """The tree path's tables for this chunk, or None when nothing is worth stacking."""
        seqs = host["seqs"]
        decode = set(host["dseqs"].tolist())
        # each prefill sequence stacks at most one earlier segment: the longest one that another
        # sequence of the chunk reads too (a shared prefix, a join anchor)
        count: dict = {}
        for si, s in enumerate(specs):
            if si not in decode and not s.bidirectional:
                for r in s.reads:
                    if r[1] >= self.tree_min_tokens:
                        count[r] = count.get(r, 0) + 1
        groups: dict = {}
        for si, s in enumerate(specs):
            if si in decode or s.bidirectional:
                continue
            best = None
            for i, r in enumerate(s.reads):
                if count.get(r, 0) >= 2 and (best is None or r[1] > s.reads[best][1]):
                    best = i
            if best is not None:
                groups.setdefault(s.reads[best], []).append((si, best))
        chosen = []
        for (key, ln), members in groups.items():
            if len(members) < 2:
                continue
            rows = [int(seqs[si, 1]) for si, _ in members]
            if self.tree == "auto" and not tree_saves(rows, ln):
                continue
            chosen.append((ln, members))
        if not chosen:
            return None
        T = host["ids"].size
        a = seqs.copy()
        b_rows, b_seqs, stacked = [], [], 0
        source = np.full(T, -1, dtype=np.int32)
        for ln, members in chosen:
            start = stacked
            for si, seg in members:
                # drop segment `seg` from the sequence's table (the own segment stays last)
                nseg = int(a[si, 2])
                lens = [int(x) for i, x in enumerate(seqs[si, 4:4 + nseg]) if i != seg]
                offs = [int(x) for i, x in enumerate(seqs[si, 8:8 + nseg]) if i != seg]
                a[si, 4:8] = 0
                a[si, 8:12] = 0
                a[si, 4:4 + nseg - 1] = lens
                a[si, 8:8 + nseg - 1] = offs
                a[si, 2] = nseg - 1
                q0, n = int(seqs[si, 0]), int(seqs[si, 1])
                r = np.arange(q0, q0 + n, dtype=np.int32)
                b_rows.append(r)
                source[r] = np.arange(stacked, stacked + n, dtype=np.int32)
                stacked += n
            si0, seg0 = members[0]
            # the stacked rows read the shared segment whole (bit 0: both ways)
            b_seqs.append([start, stacked - start, 1, 1, ln, 0, 0, 0, int(seqs[si0, 8 + seg0]), 0, 0, 0])
        seqs_b = np.asarray(b_seqs, dtype=np.int32).reshape(-1, SEQ_INTS)

        def blocks_of(tab, skip):
            out = []
            for si in range(tab.shape[0]):
                if si in skip:
                    continue
                n, nseg = int(tab[si, 1]), int(tab[si, 2])
                keys = int(tab[si, 4:4 + nseg].sum())
                for q0 in range(0, n, TREE_BLOCK):
                    out.append((keys, si, q0))
            out.sort(key=lambda x: -x[0])
            return np.asarray([(x[1], x[2]) for x in out], dtype=np.int32).reshape(-1, 2)
        return {"seqs_a": a, "seqs_b": seqs_b, "blocks_a": blocks_of(a, decode), "blocks_b": blocks_of(seqs_b, ()),
                "rows": np.concatenate(b_rows).astype(np.int32), "source": source}

    def _upload_plain(self, flat: np.ndarray) -> torch.Tensor:
        src = torch.from_numpy(np.ascontiguousarray(flat))
        if self.device.type != "cuda":
            return src.clone()
        return src.pin_memory().to(self.device, non_blocking=True) if self.pin else src.to(self.device)

    def _upload(self, flat: np.ndarray) -> torch.Tensor:
        src = torch.from_numpy(flat)
        if self.device.type != "cuda":
            return src.clone()
        if not self.pin:
            return src.to(self.device)
        # two pinned staging buffers, used in turn: a buffer is refilled only
        # after the copy out of it two chunks ago has finished
        if self._staging is None:
            self._staging = [None, None]
            self._copy_done = [None, None]
            self._turn = 0
        i = self._turn
        self._turn ^= 1
        buf = self._staging[i]
        if self._copy_done[i] is not None:
            self._copy_done[i].synchronize()
        if buf is None or buf.numel() < flat.size:
            buf = torch.empty(max(flat.size, 1 << 16) * 2, dtype=torch.int32, pin_memory=True)
            self._staging[i] = buf
        stage = buf[:flat.size]
        stage.copy_(src)
        out = torch.empty(flat.size, dtype=torch.int32, device=self.device)
        out.copy_(stage, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._copy_done[i] = ev
        return out
