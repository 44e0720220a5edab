"""Paged KV arena: device K/V pools plus host-side page accounting.

Layout on the device: one tensor [layers, 2, pages, page_tokens, kv_heads,
head_dim] bf16, so a layer's K or V pool is a contiguous view
[pages, page_tokens, kv_heads, head_dim] (the layout the K4 KV-write and K6
attention kernels take). A B200 holds 180 GB of HBM3e; the arena is sized by
the planner's `arena_pages` from what is left after weights and activations.

Accounting (`PagePool`, pure Python, CPU-testable): a free stack, page lists
per key, and a hold count per page. A key owns the pages it writes. Another
key may read a resident key's first `tokens` tokens as one of its segments
(borrowing: a question reads its document's pages, every row reads the one
copy of the shared instruction prefix); a borrow holds the parent's pages so
they are not freed under the reader. Retained keys stay resident after use
until evicted (KV reuse across operators).

Reference behavior: quail/backends/quail/executor/pages.py (PageArena:
free list, owned/borrowed pages, holds, retention) and arena.py (KVArena).
"""

from __future__ import annotations

from collections import OrderedDict

import numpy as np
import torch


class ArenaFullError(RuntimeError):
    """The arena cannot hold a request even when empty."""


class PagePool:
    """Page accounting; with `state_slots`, also one recurrent-state slot per key.

    Hybrid models (Gated DeltaNet layers) keep a fixed-size state per key
    instead of per-token KV: the state after the key's tokens. A reader of a
    key starts its own state from it, so borrowing holds the parent's slot
    as it holds the parent's pages.
    """

    def __init__(self, num_pages: int, page_tokens: int, state_slots: int = 0):
        self.num_pages = num_pages
        self.page_tokens = page_tokens
        self.state_slots = state_slots
        self.slot_free = list(range(state_slots - 1, -1, -1))
        self.slot_of: dict = {}          # key -> its state slot
        self.slot_holds = np.zeros(max(state_slots, 1), dtype=np.int32)
        self.slot_borrows: dict = {}     # key -> slots of the keys it reads
        self.free = list(range(num_pages - 1, -1, -1))  # stack: pop() gives the lowest id first
        self.owned: dict = {}          # key -> page ids it writes
        self.tokens: dict = {}         # key -> tokens resident
        self.holds = np.zeros(num_pages, dtype=np.int32)
        self.borrows: dict = {}        # key -> page lists it holds of the keys it reads
        self.retained: OrderedDict = OrderedDict()  # key -> None, oldest first

    # ------------------------------------------------------------ queries
    def pages_needed(self, tokens: int) -> int:
        return -(-tokens // self.page_tokens)

    @property
    def free_pages(self) -> int:
        return len(self.free)

    def resident(self, key) -> bool:
        return key in self.owned

    def pages_of(self, key) -> list[int]:
        return self.owned[key]

    # ------------------------------------------------------------ alloc / grow
    def alloc(self, key, tokens: int, capacity: int = 0):
        """Pages for `tokens` new tokens of a new key (at least `capacity` tokens
        of room, so later growth up to it needs no new pages), or None if the
        pool is short."""
        if key in self.owned:
            raise KeyError(f"{key!r} already resident")
        need = self.pages_needed(max(tokens, capacity))
        if need > len(self.free) or (self.state_slots and not self.slot_free):
            return None
        pages = [self.free.pop() for _ in range(need)]
        if self.state_slots:
            slot = self.slot_free.pop()
            self.slot_of[key] = slot
            self.slot_holds[slot] += 1
            self.slot_borrows[key] = []
        self.owned[key] = pages
        self.tokens[key] = tokens
        self.holds[pages] += 1
        self.borrows[key] = []
        return pages

    def grow(self, key, tokens: int):
        """Extend a resident key to `tokens` tokens; returns the new pages or None."""
        have = self.owned[key]
        need = -(-tokens // self.page_tokens) - len(have)
        if need <= 0:
            if tokens > self.tokens[key]:
                self.tokens[key] = tokens
            return []
        if need > len(self.free):
            return None
        new = [self.free.pop() for _ in range(max(need, 0))]
        have.extend(new)
        if new:
            self.holds[new] += 1
        self.tokens[key] = max(self.tokens[key], tokens)
        return new

    def borrow(self, reader, parent) -> None:
        """`reader` reads `parent`'s pages: hold them until the reader is freed."""
        if parent not in self.owned:
            raise KeyError(f"borrow parent {parent!r} is not resident")
        pages = list(self.owned[parent])
        self.holds[pages] += 1
        self.borrows.setdefault(reader, []).append(pages)
        if self.state_slots:
            slot = self.slot_of[parent]
            self.slot_holds[slot] += 1
            self.slot_borrows.setdefault(reader, []).append(slot)

    # ------------------------------------------------------------ release
    def _drop(self, pages) -> None:
        if not pages:
            return
        self.holds[pages] -= 1
        for p in pages:
            if self.holds[p] == 0:
                self.free.append(p)

    def _drop_slot(self, slot: int) -> None:
        self.slot_holds[slot] -= 1
        if self.slot_holds[slot] == 0:
            self.slot_free.append(slot)

    def free_key(self, key) -> None:
        """Release a key's own pages and the holds it took on borrowed parents."""
        for pages in self.borrows.pop(key, []):
            self._drop(pages)
        for slot in self.slot_borrows.pop(key, []):
            self._drop_slot(slot)
        if key in self.slot_of:
            self._drop_slot(self.slot_of.pop(key))
        pages = self.owned.pop(key, None)
        self.tokens.pop(key, None)
        self.retained.pop(key, None)
        if pages is not None:
            self._drop(pages)

    def rewind(self, key, tokens: int) -> None:
        """Trim a resident key back to its first `tokens` tokens and release the pages past them
        (pages a reader still holds stay held until it is freed)."""
        have = self.owned[key]
        keep = self.pages_needed(tokens)
        if keep < len(have):
            self._drop(have[keep:])
            del have[keep:]
        self.tokens[key] = min(self.tokens[key], tokens)

    def adopt(self, old, new) -> None:
        """Give a resident key's pages, holds and state slot to a new key (no longer retained)."""
        if new in self.owned:
            raise KeyError(f"{new!r} already resident")
        self.owned[new] = self.owned.pop(old)
        self.tokens[new] = self.tokens.pop(old)
        self.borrows[new] = self.borrows.pop(old, [])
        if old in self.slot_of:
            self.slot_of[new] = self.slot_of.pop(old)
            self.slot_borrows[new] = self.slot_borrows.pop(old, [])
        self.retained.pop(old, None)

    def retain(self, key) -> None:
        self.retained[key] = None
        self.retained.move_to_end(key)

    def evict_retained(self, pages_needed: int) -> list:
        """Free retained keys, oldest first, until `pages_needed` pages are free."""
        evicted = []
        while self.free_pages < pages_needed and self.retained:
            key, _ = self.retained.popitem(last=False)
            self.free_key(key)
            evicted.append(key)
        return evicted

    def check(self) -> None:
        """Invariant: every page is free xor held; holds match owners and borrows."""
        expect = np.zeros(self.num_pages, dtype=np.int32)
        for pages in self.owned.values():
            expect[pages] += 1
        for held in self.borrows.values():
            for pages in held:
                expect[pages] += 1
        assert np.array_equal(expect, self.holds), "hold counts drifted"
        free = set(self.free)
        assert len(free) == len(self.free), "page freed twice"
        for p in range(self.num_pages):
            assert (p in free) == (self.holds[p] == 0), f"page {p} free/held mismatch"
        if self.state_slots:
            want = np.zeros(self.state_slots, dtype=np.int32)
            for slot in self.slot_of.values():
                want[slot] += 1
            for slots in self.slot_borrows.values():
                for slot in slots:
                    want[slot] += 1
            assert np.array_equal(want, self.slot_holds[:self.state_slots]), "state slot holds drifted"
            sf = set(self.slot_free)
            assert len(sf) == len(self.slot_free), "state slot freed twice"
            for q in range(self.state_slots):
                assert (q in sf) == (want[q] == 0), f"state slot {q} free/held mismatch"


class KVArena:
    """Device K/V pools with a PagePool."""

    def __init__(self, num_layers: int, num_pages: int, page_tokens: int, kv_heads: int, head_dim: int,
                 device="cuda", dtype=torch.bfloat16, state_slots: int = 0, state_shapes: dict | None = None,
                 layer_geoms: list | None = None):
        self.num_layers = num_layers
        self.page_tokens = page_tokens
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        self.device = torch.device(device)
        # layers of another (KV heads, head_dim) (Gemma 4's global layers) get a pool tensor of
        # their own, addressed by the same page ids
        geoms = list(layer_geoms) if layer_geoms else [(kv_heads, head_dim)] * num_layers
        assert len(geoms) == num_layers
        self._where = []
        count: dict = {}
        for g in geoms:
            self._where.append((g, count.get(g, 0)))
            count[g] = count.get(g, 0) + 1
        self.groups = {g: torch.zeros(n, 2, num_pages, page_tokens, g[0], g[1], device=device, dtype=dtype)
                       for g, n in count.items()}
        self.kv = self.groups.get((kv_heads, head_dim), next(iter(self.groups.values())))
        self.pool = PagePool(num_pages, page_tokens, state_slots)
        # recurrent states of hybrid models: name -> [slots, *shape] fp32 (e.g. conv window, delta-rule state)
        self.states = {name: torch.zeros(state_slots, *shape, device=device, dtype=torch.float32)
                       for name, shape in (state_shapes or {}).items()}

    @classmethod
    def for_model(cls, cfg, num_pages: int, page_tokens: int, device="cuda", dtype=torch.bfloat16,
                  state_slots: int = 0) -> "KVArena":
        """KV pages for the model's attention layers; state slots for its Gated DeltaNet layers."""
        shapes = None
        if cfg.is_hybrid:
            shapes = {}
            G = len(cfg.gdn_layers)
            if G:
                shapes["conv"] = (G, cfg.conv_width - 1, cfg.gdn_conv_dim)
                shapes["ssm"] = (G, cfg.gdn_value_heads, cfg.gdn_key_dim, cfg.gdn_value_dim)
            if cfg.conv_layers:
                shapes["sconv"] = (len(cfg.conv_layers), cfg.conv_width - 1, cfg.hidden)
            state_slots = state_slots or 64
        geoms = [cfg.attn_geometry(i) for i in cfg.attn_layers] if getattr(cfg, "gemma4", False) else None
        return cls(len(cfg.attn_layers), num_pages, page_tokens, cfg.num_kv_heads, cfg.head_dim, device=device,
                   dtype=dtype, state_slots=state_slots if cfg.is_hybrid else 0, state_shapes=shapes,
                   layer_geoms=geoms)

    @property
    def num_pages(self) -> int:
        return self.pool.num_pages

    def layer(self, i: int):
        g, j = self._where[i]
        t = self.groups[g]
        return t[j, 0], t[j, 1]

    @staticmethod
    def bytes_per_page(num_layers, page_tokens, kv_heads, head_dim, elem_bytes=2) -> int:
        return num_layers * 2 * page_tokens * kv_heads * head_dim * elem_bytes
