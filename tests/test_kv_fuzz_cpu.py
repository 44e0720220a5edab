"""KV-correctness fuzz: the real executor, packer and arena on CPU with a hashing model.

The model stores each new token's (id, position) in its KV slot and answers a
read row with a hash of every token the row can see, gathered through the
chunk's segments and page list. A wrong page, a stale or trimmed segment, a
reused borrowed page or a wrong position gives a hash no prompt has (positions
out of order give NaN). Random corpora with a shared prefix, documents read by
several questions (borrowed pages), small chunks (prefill split into pieces),
decode continuations and a tiny arena (eviction, admission under pressure) run
against the hashes of the plain prompts.

Reference: tests/helpers/kv_checker.py (HashModel) of the reference.
"""

import numpy as np
import pytest
import torch

from quail_b200.engine.arena import KVArena
from quail_b200.engine.stage_executor import StageExecutor, Task

MOD = 2_147_483_629


def prompt_hash(tokens) -> float:
    h = 17
    for t in tokens:
        h = (h * 1_000_003 + int(t) + 1) % MOD
    return float(h)


class HashModel:
    """forward_chunk writes (id, position) into the KV slots and hashes what each read row sees."""

    def forward_chunk(self, chunk, arena):
        kc, _ = arena.layer(0)
        kc = kc.reshape(-1, kc.shape[-2], kc.shape[-1])        # [slot, kv head, d]
        P = arena.pool.page_tokens
        h = chunk.host
        ids, pos, slots, seqs, pl = h["ids"], h["positions"], h["slots"], h["seqs"], h["page_list"]
        for t in range(ids.size):
            if slots[t] >= 0:
                kc[slots[t], 0, 0] = float(ids[t])
                kc[slots[t], 0, 1] = float(pos[t])
        want_rows = {int(r) for r in h["final_rows"]}
        value = {}
        for row in seqs:
            q0, n, nseg = int(row[0]), int(row[1]), int(row[2])
            toks, posl = [], []
            for i in range(nseg):
                ln, off = int(row[4 + i]), int(row[8 + i])
                pages = pl[off:off + -(-ln // P)]
                sl = [int(pages[j // P]) * P + j % P for j in range(ln)]
                toks.append(kc[sl, 0, 0].numpy())
                posl.append(kc[sl, 0, 1].numpy())
            seen = np.concatenate(toks) if toks else np.zeros(0)
            seen_pos = np.concatenate(posl) if posl else np.zeros(0)
            own_len = int(row[4 + nseg - 1])
            before = len(seen) - own_len                 # tokens of the segments read in full
            for k in range(n):
                r = q0 + k
                if r not in want_rows:
                    continue
                upto = before + own_len - n + k + 1      # the row sees the new tokens up to itself
                ok = np.array_equal(seen_pos[:upto], np.arange(upto))
                value[r] = prompt_hash(seen[:upto]) if ok else float("nan")
        return torch.tensor([[value[int(r)]] for r in h["final_rows"]], dtype=torch.float64)


@pytest.mark.parametrize("seed,pages,page_tokens,chunk", [(0, 40, 4, 24), (1, 24, 8, 64), (2, 60, 4, 9),
                                                          (3, 14, 16, 128)])
def test_every_read_row_sees_its_prompt(seed, pages, page_tokens, chunk):
    rng = np.random.default_rng(seed)
    arena = KVArena(1, pages, page_tokens, 1, 2, device="cpu", dtype=torch.float64)
    ex = StageExecutor(HashModel(), arena, chunk, min_piece=2)
    prefix = rng.integers(0, 500, int(rng.integers(1, 12))).astype(np.int32)
    docs = [rng.integers(0, 500, int(rng.integers(1, 40))).astype(np.int32) for _ in range(12)]
    questions = [rng.integers(0, 500, int(rng.integers(1, 6))).astype(np.int32) for _ in range(3)]
    want, got = {}, {}
    P = len(prefix)
    ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))

    def doc_done(i, row):
        got[("d", i)] = float(row[0])
        # the document's other questions read its pages (borrowed), then a decode step continues one
        for qi, q in enumerate(questions[1:], start=1):
            key = ("q", i, qi)
            want[key] = prompt_hash(np.concatenate([prefix, docs[i], q]))
            ex.submit(Task(key=key, tokens=q, pos_start=P + len(docs[i]), reads=[("p", P), (("d", i), len(docs[i]))],
                           readout=True, free_after=False,
                           on_done=lambda t, r, key=key, q=q: step(key, q, r)))

    pending = {i: len(questions) - 1 for i in range(len(docs))}

    def last_done(k2, i, row):
        # the decode step frees its question (free_after); the document goes with its last question
        got[k2] = float(row[0])
        pending[i] -= 1
        if pending[i] == 0:
            ex.free(("d", i))

    def step(key, q, row):
        got[key] = float(row[0])
        i = key[1]
        extra = np.array([7], dtype=np.int32)
        k2 = key + ("next",)
        want[k2] = prompt_hash(np.concatenate([prefix, docs[i], q, extra]))
        ex.submit(Task(key=key, tokens=extra, pos_start=P + len(docs[i]) + len(q),
                       reads=[("p", P), (("d", i), len(docs[i]))], readout=True, own_prefix=len(q),
                       on_done=lambda t, r, k2=k2, i=i: last_done(k2, i, r)))

    for i, d in enumerate(docs):
        toks = np.concatenate([d, questions[0]])
        want[("d", i)] = prompt_hash(np.concatenate([prefix, toks]))
        ex.submit(Task(key=("d", i), tokens=toks, pos_start=P, reads=[("p", P)], readout=True, free_after=False,
                       on_done=lambda t, r, i=i: doc_done(i, r)))
    ex.run()
    assert set(got) == set(want)
    bad = {k: (got[k], want[k]) for k in want if got[k] != want[k]}
    assert not bad, list(bad.items())[:3]
    ex.free("p")
    assert arena.pool.free_pages == arena.pool.num_pages
    arena.pool.check()
