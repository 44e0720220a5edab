"""CUDA graphs of decode passes: one captured forward per token bucket.

A decode pass (every sequence of the chunk has one new token, as in AI.MAP
and AI.EXTRACT's greedy steps) is a few hundred small kernel launches over
few rows, so the host's launch cost, not the GPU, sets its time. Such a pass
runs as the replay of a graph captured for the smallest bucket B >= its
token count (buckets 8, 16, 32, 64, 128, 256, 512, 1024):

  * each bucket owns one device int32 buffer laid out as a chunk of B
    one-token sequences (ids, positions, slots, seqs, page list capacity,
    final rows, dseqs), so the captured kernels read fixed addresses;
  * a pass fills the buffer's host image (its real rows, then padding rows:
    token 0, no KV slot (-1, the write is skipped), one own segment of one
    token on the arena's page 0, read and discarded, and for hybrid models
    no state slot (state_io -1, -1: it starts from zeros and its state is
    not written back)), copies it with one H2D copy and replays the graph;
  * the first pass of a bucket runs eagerly (its result is the pass's) and
    then captures; a page list longer than the bucket's capacity recaptures
    with twice the capacity; new answer rows (another query) drop the graphs.

Every bucket's graph allocates from one shared memory pool (they replay one
at a time on one stream), and the logits a replay returns live in that pool
until the next replay, after the executor's D2H copy on the same stream.

Reference: quail/backends/quail/executor/cuda_graphs.py:16-428 (piecewise
graphs split at the token mixers, token buckets) and warmup.py. Here the
whole forward of a decode pass is one graph: the attention kernels read
their per-sequence work from device metadata, so nothing in the pass
depends on host values but the bucket size.
"""

from __future__ import annotations

import numpy as np
import torch

from quail_b200.engine.chunk import PARTS, SEQ_INTS, Chunk

BUCKETS = (8, 16, 32, 64, 128, 256, 512, 1024)


class _Entry:
    def __init__(self, B: int, pl_cap: int, device):
        self.B = B
        self.pl_cap = pl_cap
        self.sizes = {"ids": B, "positions": B, "slots": B, "seqs": B * SEQ_INTS, "tiles": 0,
                      "page_list": pl_cap + 1, "final_rows": B, "dseqs": B, "state_io": 2 * B,
                      "blocks": 0}
        self.total = sum(self.sizes.values())
        self.buf = torch.zeros(self.total, dtype=torch.int32, device=device)
        # two pinned staging images, used in turn: filling one waits only for the copy out of
        # the other two passes back, so the host stays a pass ahead of the replays (with one
        # image it waited for the previous pass's copy, which is queued behind its replay)
        self.stages = [torch.empty(self.total, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self.copies = [None, None]
        self.turn = 0
        self.graph = None
        self.out = None
        self.launches = 0

    def chunk(self, full: bool, topk: bool = False) -> Chunk:
        v, o = {}, 0
        for k in PARTS:
            v[k] = self.buf[o:o + self.sizes[k]]
            o += self.sizes[k]
        return Chunk(num_tokens=self.B, ids=v["ids"], positions=v["positions"], slots=v["slots"],
                     seqs=v["seqs"].view(-1, SEQ_INTS), tiles=v["tiles"].view(-1, 2), page_list=v["page_list"],
                     final_rows=v["final_rows"], dseqs=v["dseqs"], state_io=v["state_io"].view(-1, 2),
                     blocks=v["blocks"].view(-1, 2), num_seqs=self.B, full_readout=full, topk=topk)

    def fill(self, host: dict) -> int:
        """Write a pass's metadata, padded to the bucket, into the staging image; returns its bytes."""
        B, T = self.B, host["ids"].size
        pl = host["page_list"]
        img = {
            "ids": np.zeros(B, np.int32), "positions": np.zeros(B, np.int32),
            "slots": np.full(B, -1, np.int32), "seqs": np.zeros((B, SEQ_INTS), np.int32),
            "tiles": np.zeros(0, np.int32), "page_list": np.zeros(self.pl_cap + 1, np.int32),
            "final_rows": np.arange(B, dtype=np.int32), "dseqs": np.arange(B, dtype=np.int32),
            "state_io": np.full((B, 2), -1, np.int32), "blocks": np.zeros(0, np.int32),
        }
        for k in ("ids", "positions", "slots"):
            img[k][:T] = host[k]
        img["seqs"][:T] = host["seqs"]
        pad = img["seqs"][T:]
        pad[:, 0] = np.arange(T, B)     # q_start: its own row
        pad[:, 1] = 1                   # one query token
        pad[:, 2] = 1                   # one segment (its own)
        pad[:, 4] = 1                   # of one token
        pad[:, 8] = self.pl_cap         # on the page at the last page-list entry (page 0)
        img["page_list"][:pl.size] = pl
        img["final_rows"][:host["final_rows"].size] = host["final_rows"]
        if "state_io" in host:
            # hybrid models: real rows carry their state slots; padding starts from zeros and keeps nothing
            img["state_io"][:T] = np.asarray(host["state_io"]).reshape(-1, 2)[:T]
        flat = np.concatenate([img[k].reshape(-1) for k in PARTS])
        i = self.turn
        self.turn ^= 1
        if self.copies[i] is not None:
            self.copies[i].synchronize()
        self.stages[i].copy_(torch.from_numpy(flat))
        self.buf.copy_(self.stages[i], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.copies[i] = ev
        return int(flat.nbytes)


class DecodeGraphs:
    """Replays captured decode passes of `model` (a pipeline with forward_chunk) over `arena`."""

    def __init__(self, model, arena, device, buckets=BUCKETS):
        self.model = model
        self.arena = arena
        self.device = torch.device(device)
        self.buckets = tuple(buckets)
        self.entries: dict = {}
        self.pool = torch.cuda.graph_pool_handle()
        self._rows_key = None
        self.replays = 0
        self.captures = 0

    @staticmethod
    def eligible(specs) -> bool:
        """A pass of one-token sequences, each read out at its token (or not at all)."""
        return bool(specs) and all(len(s.tokens) == 1 and s.readout_rows is None for s in specs)

    def _answer_key(self):
        w = getattr(self.model, "w", self.model)
        rows = getattr(w, "answer_rows", None)
        return None if rows is None else (rows.data_ptr(), tuple(rows.shape))

    def bucket(self, n: int) -> int | None:
        for b in self.buckets:
            if n <= b:
                return b
        return None

    def run(self, host: dict, full: bool, topk: bool = False):
        """Run one decode pass from its host metadata; returns (readout rows [R, W], upload bytes)
        or None when the pass has no bucket (too many tokens)."""
        from quail_b200 import ops
        T = host["ids"].size
        B = self.bucket(T)
        if B is None:
            return None
        key = self._answer_key()
        if key != self._rows_key:
            self.entries.clear()
            self._rows_key = key
        pl_need = host["page_list"].size
        e = self.entries.get((B, full, topk))
        if e is not None and pl_need > e.pl_cap:
            e = None
        if e is None:
            cap = 1 << max(10, int(np.ceil(np.log2(max(pl_need, 1)))) + 1)
            e = _Entry(B, cap, self.device)
            self.entries[(B, full, topk)] = e
        nbytes = e.fill(host)
        R = host["final_rows"].size
        if e.graph is None:
            chunk = e.chunk(full, topk)
            out = self.model.forward_chunk(chunk, self.arena)      # eager: this pass's answer
            torch.cuda.current_stream().synchronize()
            n0 = ops.launch_count()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.pool):
                e.out = self.model.forward_chunk(chunk, self.arena)
            e.launches = ops.launch_count() - n0
            ops.count_launch(-e.launches)        # capture launched nothing
            e.graph = g
            self.captures += 1
            return out[:R], nbytes
        e.graph.replay()
        ops.count_launch(e.launches)
        self.replays += 1
        return e.out[:R], nbytes

    def clear(self) -> None:
        self.entries.clear()
