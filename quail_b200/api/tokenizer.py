"""Tokenizers: the model's own (HF tokenizer.json) or a self-contained byte-level one.

A model loaded from a checkpoint directory uses the `tokenizer.json` beside
the weights (byte-level BPE, read by `tokenizers`). Random-init models, and
the tests, use `ByteTokenizer`: one id per UTF-8 byte plus the chat special
tokens, so prompts tokenize the same on every machine without downloads.
"""

from __future__ import annotations

import os

import numpy as np

SPECIALS = ("<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>")


class ByteTokenizer:
    """id = 256 + byte for text; specials at 0..4; answer words get ids of their own."""

    def __init__(self, vocab: int = 151_936):
        self.vocab = vocab
        self.special = {s: i for i, s in enumerate(SPECIALS)}
        self.eos_ids = (self.special["<|im_end|>"], self.special["<|endoftext|>"])

    def encode(self, text: str) -> np.ndarray:
        out: list[int] = []
        i, n = 0, len(text)
        while i < n:
            if text[i] == "<":
                for s, sid in self.special.items():
                    if text.startswith(s, i):
                        out.append(sid)
                        i += len(s)
                        break
                else:
                    out.extend(256 + b for b in text[i].encode("utf-8"))
                    i += 1
            else:
                j = text.find("<", i)
                j = n if j < 0 else j
                out.extend(256 + b for b in text[i:j].encode("utf-8"))
                i = j
        return np.asarray(out, dtype=np.int32)

    def decode(self, ids) -> str:
        inv = {v: k for k, v in self.special.items()}
        parts, buf = [], bytearray()
        for t in ids:
            t = int(t)
            if t in inv:
                if buf:
                    parts.append(buf.decode("utf-8", errors="replace"))
                    buf = bytearray()
                parts.append(inv[t])
            elif 256 <= t < 512:
                buf.append(t - 256)
        if buf:
            parts.append(buf.decode("utf-8", errors="replace"))
        return "".join(parts)

    def token_id(self, word: str) -> int | None:
        ids = self.encode(word)
        return int(ids[0]) if len(ids) == 1 else None

    def answer_ids(self, spellings) -> list[int]:
        """First token of each answer spelling (deduplicated, order kept)."""
        out = []
        for s in spellings:
            ids = self.encode(s)
            if len(ids) and int(ids[0]) not in out:
                out.append(int(ids[0]))
        return out


class HFTokenizer:
    """A Hugging Face tokenizer.json (byte-level BPE) through the `tokenizers` library."""

    def __init__(self, path: str):
        from tokenizers import Tokenizer
        if os.path.isdir(path):
            path = os.path.join(path, "tokenizer.json")
        self.tok = Tokenizer.from_file(path)
        self.vocab = self.tok.get_vocab_size()
        ids = [self.tok.token_to_id(s) for s in ("<|im_end|>", "<|endoftext|>")]
        self.eos_ids = tuple(i for i in ids if i is not None)

    def encode(self, text: str) -> np.ndarray:
        return np.asarray(self.tok.encode(text, add_special_tokens=False).ids, dtype=np.int32)

    def decode(self, ids) -> str:
        return self.tok.decode([int(i) for i in ids], skip_special_tokens=False)

    def token_id(self, word: str):
        return self.tok.token_to_id(word)

    def answer_ids(self, spellings) -> list[int]:
        out = []
        for s in spellings:
            ids = self.encode(s)
            if len(ids) and int(ids[0]) not in out:
                out.append(int(ids[0]))
        return out


QWEN2_SPLIT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"
               r"|\s*[\r\n]+|\s+(?!\S)|\s+")


def _native_compatible(spec: dict) -> bool:
    """True when the tokenizer.json is the byte-level BPE the native tokenizer implements."""
    model = spec.get("model") or {}
    if model.get("type") != "BPE" or model.get("dropout") or model.get("continuing_subword_prefix"):
        return False
    norm = spec.get("normalizer")
    if norm is not None and norm.get("type") != "NFC":
        return False
    pre = spec.get("pre_tokenizer") or {}
    steps = pre.get("pretokenizers", []) if pre.get("type") == "Sequence" else [pre]
    if len(steps) != 2:
        return False
    split, byte = steps
    pattern = (split.get("pattern") or {}).get("Regex")
    return (split.get("type") == "Split" and pattern == QWEN2_SPLIT and split.get("behavior") == "Isolated"
            and byte.get("type") == "ByteLevel" and not byte.get("add_prefix_space")
            and not byte.get("use_regex", True))


class NativeBpeTokenizer:
    """A byte-level BPE tokenizer.json (Qwen2 pre-tokenizer) on the C++ tokenizer.

    Encoding runs in native code with the GIL released (`encode_batch` takes
    a whole column), merges are cached per pre-token. The NFC normalizer is
    applied here, in Python, before the native split.
    Reference: crates/quail/src/inputs/tokenizer.rs (the reference's batch
    tokenization through the `tokenizers` crate).
    """

    def __init__(self, path: str, spec: dict | None = None):
        import json
        from quail_b200 import _native
        if os.path.isdir(path):
            path = os.path.join(path, "tokenizer.json")
        if spec is None:
            with open(path, encoding="utf-8") as f:
                spec = json.load(f)
        model = spec["model"]
        merges = [tuple(m.split(" ", 1)) if isinstance(m, str) else tuple(m) for m in model.get("merges", [])]
        added = {a["content"]: int(a["id"]) for a in spec.get("added_tokens", [])}
        self.nfc = spec.get("normalizer") is not None
        self.tok = _native.BpeTokenizer(model["vocab"], merges, added, bool(model.get("ignore_merges", False)))
        self.vocab = self.tok.vocab_size
        ids = [self.tok.token_to_id(s) for s in ("<|im_end|>", "<|endoftext|>")]
        self.eos_ids = tuple(i for i in ids if i >= 0)

    def _norm(self, text: str) -> str:
        if self.nfc and not text.isascii():
            import unicodedata
            return unicodedata.normalize("NFC", text)
        return text

    def encode(self, text: str) -> np.ndarray:
        return np.asarray(self.tok.encode(self._norm(text)), dtype=np.int32)

    def encode_batch(self, texts) -> list[np.ndarray]:
        return [np.asarray(r, dtype=np.int32) for r in self.tok.encode_batch([self._norm(t) for t in texts])]

    def decode(self, ids) -> str:
        return self.tok.decode([int(i) for i in ids], False).decode("utf-8", errors="replace")

    def token_id(self, word: str):
        i = self.tok.token_to_id(word)
        return None if i < 0 else i

    def answer_ids(self, spellings) -> list[int]:
        out = []
        for s in spellings:
            ids = self.encode(s)
            if len(ids) and int(ids[0]) not in out:
                out.append(int(ids[0]))
        return out


class WordTokenizer(ByteTokenizer):
    """One token per word or punctuation mark, id from a stable hash of its text.

    Lengths come out close to a BPE tokenizer's on English text, which makes
    it the tokenizer of the synthetic benchmark tables; decode() is not
    available (hashes do not invert), so it is not for AI.MAP output.
    """

    def __init__(self, vocab: int = 151_936):
        super().__init__(vocab)
        import re
        self._split = re.compile(r"<\|[a-z_]+\|>|</?think>|\s*[A-Za-z0-9]+|\s*[^\sA-Za-z0-9]|\s+")

    def encode(self, text: str) -> np.ndarray:
        import zlib
        out = []
        for m in self._split.finditer(text):
            piece = m.group(0)
            sid = self.special.get(piece.strip()) if piece.strip() in self.special else None
            out.append(sid if sid is not None else 1024 + zlib.crc32(piece.encode()) % (self.vocab - 1024))
        return np.asarray(out, dtype=np.int32)

    def decode(self, ids) -> str:
        return " ".join(f"<{int(i)}>" for i in ids)


def load_tokenizer(path: str | None, vocab: int):
    if path == "words":
        return WordTokenizer(vocab)
    if path is not None and os.path.exists(path if not os.path.isdir(path) else os.path.join(path, "tokenizer.json")):
        import json
        fp = os.path.join(path, "tokenizer.json") if os.path.isdir(path) else path
        with open(fp, encoding="utf-8") as f:
            spec = json.load(f)
        if _native_compatible(spec) and os.environ.get("QB_HF_TOKENIZER") != "1":
            try:
                return NativeBpeTokenizer(fp, spec)
            except ImportError:
                pass
        return HFTokenizer(path)
    return ByteTokenizer(vocab)
