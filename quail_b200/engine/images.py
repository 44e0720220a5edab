"""Image documents: pixels in, image tokens out, their embeddings from the vision tower.

An image document becomes the vision start token, one token per 32 x 32 pixels
(row by row) and the vision end token. An image token's id is
IMAGE_TOKEN_BASE + the image's first token index + its index in the image, so a
token array names its images' tokens without a side table; the store keeps each
image's geometry and pixels, runs the vision tower on a region's images before
its passes, and gives every image token its embedding row.

Positions (Qwen's multimodal RoPE): an image whose first token sits at rotary
position s gives its token at row i, column j the positions (s, s + i, s + j)
(time, height, width) and the next token the position s + max(rows, columns),
so the rotary positions of everything after an image run behind the KV
positions by tokens - max(rows, columns). `rope_positions` computes the three
streams of a packed sequence from its tokens, its KV positions and the shift
its earlier segments carry (the reference's RegionImages.rotary_positions,
quail/backends/quail/executor/images.py:238-313).
"""

from __future__ import annotations

import bisect
import io
from dataclasses import dataclass

import numpy as np
import torch

IMAGE_TOKEN_BASE = 1 << 28
# the longer side an image is read at when its document does not say (pixels)
DEFAULT_LONGEST = 1024


@dataclass
class Image:
    first: int                  # index of its first token among the store's image tokens
    rows: int
    cols: int
    pixels: torch.Tensor        # [3, rows * 32, cols * 32] normalized

    @property
    def tokens(self) -> int:
        return self.rows * self.cols

    @property
    def shift(self) -> int:
        """How much less the rotary positions after the image advance than its tokens."""
        return self.tokens - max(self.rows, self.cols)


def decode_rgb(data: bytes) -> np.ndarray:
    """PNG / JPEG bytes -> uint8 [H, W, 3]."""
    from PIL import Image as PILImage
    im = PILImage.open(io.BytesIO(data)).convert("RGB")
    return np.asarray(im)


class ImageStore:
    """The images of a model engine's regions and their token embeddings."""

    def __init__(self, cfg, longest: int = DEFAULT_LONGEST):
        self.cfg = cfg
        self.longest = longest
        self.images: list[Image] = []
        self._firsts: list[int] = []
        self.next = 0
        self._table: torch.Tensor | None = None     # embeddings of images [0, encoded)
        self._encoded = 0
        self._seen: dict = {}                        # encoded bytes -> their tokens (one read per image)

    def add(self, data) -> np.ndarray:
        """Register an image (encoded bytes or uint8 [H, W, 3]); its document's token ids."""
        from PIL import Image as PILImage

        from quail_b200.models.vision import image_size, pixels, token_pixels
        key = bytes(data) if isinstance(data, (bytes, bytearray, memoryview)) else None
        if key is not None and key in self._seen:
            return self._seen[key]
        rgb = decode_rgb(data) if key is not None else np.asarray(data, np.uint8)
        h, w = rgb.shape[:2]
        cols, rows = image_size(w, h, self.longest, self.cfg)
        px = token_pixels(self.cfg)
        if (w, h) != (cols * px, rows * px):
            rgb = np.asarray(PILImage.fromarray(rgb).resize((cols * px, rows * px), PILImage.BICUBIC))
        img = Image(first=self.next, rows=rows, cols=cols, pixels=pixels(rgb))
        self.images.append(img)
        self._firsts.append(img.first)
        self.next += img.tokens
        ids = IMAGE_TOKEN_BASE + img.first + np.arange(img.tokens, dtype=np.int64)
        out = np.concatenate([[self.cfg.vision_start_id], ids, [self.cfg.vision_end_id]]).astype(np.int32)
        if key is not None:
            self._seen[key] = out
        return out

    def find(self, offset: int) -> Image:
        """The image holding image-token index `offset`."""
        return self.images[bisect.bisect_right(self._firsts, offset) - 1]

    def encode(self, tower) -> int:
        """Run the vision tower on the images not encoded yet; returns how many it ran."""
        todo = [im for im in self.images if im.first >= self._encoded]
        if not todo:
            return 0
        outs = tower.encode([im.pixels for im in todo])
        new = torch.cat(outs)
        self._table = new if self._table is None else torch.cat([self._table, new.to(self._table.device)])
        self._encoded = self.next
        return len(todo)

    def table(self, device, dtype) -> torch.Tensor:
        t = self._table
        if t is None or t.shape[0] < self.next:
            raise RuntimeError("image tokens read before their images were encoded")
        if t.device != torch.device(device) or t.dtype != dtype:
            self._table = t = t.to(device=device, dtype=dtype)
        return t

    def clear(self) -> None:
        self.images.clear()
        self._firsts.clear()
        self.next = 0
        self._table = None
        self._encoded = 0
        self._seen.clear()

    def rope_positions(self, tokens: np.ndarray, kv_pos: np.ndarray, shift: int) -> tuple[np.ndarray, int]:
        """[n, 3] rotary positions of a sequence's tokens and the shift after them."""
        tokens = np.asarray(tokens, dtype=np.int64)
        base = np.asarray(kv_pos, dtype=np.int64) - shift
        out = np.repeat(base[:, None], 3, axis=1)
        where = np.nonzero(tokens >= IMAGE_TOKEN_BASE)[0]
        if where.size == 0:
            return out.astype(np.int32), shift
        offs = tokens[where] - IMAGE_TOKEN_BASE
        i = 0
        while i < where.size:
            img = self.find(int(offs[i]))
            j = i
            while j < where.size and img.first <= offs[j] < img.first + img.tokens:
                j += 1
            idx, k = where[i:j], offs[i:j] - img.first
            s = out[idx[0], 0] - k[0]                       # rotary position of the image's first token
            out[idx, 0] = s
            out[idx, 1] = s + k // img.cols
            out[idx, 2] = s + k % img.cols
            if k[-1] == img.tokens - 1:
                # the image ends here: everything after it runs `shift` behind the KV positions
                out[idx[-1] + 1:] -= img.shift
                shift += img.shift
            i = j
        return out.astype(np.int32), shift
