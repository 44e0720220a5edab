"""Token ids of documents, kept across a session's queries.

Tokenizing is host work that repeats when queries read the same documents:
the store maps a document's text (by a 16-byte BLAKE2 digest) to its token
ids, least recently used first out once it holds more than `capacity_tokens`.
A region's documents are looked up in one pass; the misses go to the
tokenizer's batch encoder together and are stored. The planner reads lengths
from it too (`mean_tokens`), so a column tokenized once is priced by its real
lengths (the reference keeps Arrow token stores per scan for the same two
uses: crates/quail/src/planning.rs token stores, R6).
"""

from __future__ import annotations

import hashlib
from collections import OrderedDict

import numpy as np


def _key(text: str) -> bytes:
    return hashlib.blake2b(text.encode("utf-8", "surrogatepass"), digest_size=16).digest()


class TokenStore:
    def __init__(self, capacity_tokens: int = 200_000_000):
        self.capacity = capacity_tokens
        self._map: OrderedDict = OrderedDict()
        self.tokens = 0
        self.hits = 0
        self.misses = 0

    def __len__(self) -> int:
        return len(self._map)

    def get(self, text: str):
        k = _key(text)
        v = self._map.get(k)
        if v is not None:
            self._map.move_to_end(k)
            self.hits += 1
        return v

    def put(self, text: str, ids: np.ndarray) -> None:
        k = _key(text)
        if k in self._map:
            return
        ids = np.asarray(ids, dtype=np.int32)
        self._map[k] = ids
        self.tokens += ids.size
        while self.tokens > self.capacity and self._map:
            _, old = self._map.popitem(last=False)
            self.tokens -= old.size

    def encode_all(self, texts: list[str], encode_batch) -> list[np.ndarray]:
        """Token ids of every text: stored ones from the store, the rest encoded in one batch."""
        out = [None] * len(texts)
        todo: dict = {}                 # text -> the rows that wait for it (one encode per text)
        for i, t in enumerate(texts):
            v = self.get(t)
            if v is None:
                todo.setdefault(t, []).append(i)
            else:
                out[i] = v
        if todo:
            self.misses += len(todo)
            uniq = list(todo)
            for t, ids in zip(uniq, encode_batch(uniq)):
                ids = np.asarray(ids, dtype=np.int32)
                self.put(t, ids)
                for i in todo[t]:
                    out[i] = ids
        return out

    def mean_tokens(self, texts: list[str]) -> float | None:
        """Mean length of the texts the store holds among `texts` (None when it holds none)."""
        lens = [v.size for v in (self._map.get(_key(t)) for t in texts) if v is not None]
        return float(np.mean(lens)) if lens else None
