"""CPU document functions: AI.PARSE_DOCUMENT, AI.PDF_PAGES, AI.IMAGE.

The reference runs these on the CPU inside its SQL engine
(crates/quail-datafusion/src/functions/parse_document.rs, pdf_pages.rs,
image.rs). AI.PARSE_DOCUMENT here reads the text a PDF stores: it inflates
the content streams and collects the strings shown by Tj / TJ / ' / "
operators between BT and ET. AI.IMAGE shrinks an image (PNG / JPEG bytes) so
its longer side is at most `longest_edge` pixels and returns PNG bytes.
AI.PDF_PAGES(pdf [, longest_edge [, first [, last]]]) draws each page as a PNG
(`sql/pdf_render.py`) and returns list<struct<page int32, image binary>>, one
entry per page, for UNNEST and a vision model.
"""

from __future__ import annotations

import io
import re
import zlib

import pyarrow as pa


def _inflate_streams(data: bytes):
    for m in re.finditer(rb"<<(.*?)>>\s*stream\r?\n", data, re.S):
        start = m.end()
        end = data.find(b"endstream", start)
        if end < 0:
            continue
        raw = data[start:end].rstrip(b"\r\n")
        if b"FlateDecode" in m.group(1):
            try:
                yield zlib.decompress(raw)
            except zlib.error:
                continue
        else:
            yield raw


def _pdf_string(s: bytes) -> str:
    out = bytearray()
    i = 0
    while i < len(s):
        c = s[i]
        if c == 0x5C and i + 1 < len(s):  # backslash escape
            n = s[i + 1]
            table = {ord("n"): 10, ord("r"): 13, ord("t"): 9, ord("b"): 8, ord("f"): 12}
            if n in table:
                out.append(table[n])
                i += 2
            elif 0x30 <= n <= 0x37:
                j = i + 1
                while j < len(s) and j < i + 4 and 0x30 <= s[j] <= 0x37:
                    j += 1
                out.append(int(s[i + 1:j], 8) & 0xFF)
                i = j
            else:
                out.append(n)
                i += 2
        else:
            out.append(c)
            i += 1
    return out.decode("latin-1")


def parse_document(data: bytes) -> str:
    if data is None:
        return None
    texts = []
    for stream in _inflate_streams(data):
        for bt in re.finditer(rb"BT(.*?)ET", stream, re.S):
            line = []
            for tok in re.finditer(rb"\((?:\\.|[^\\)])*\)|\[(.*?)\]\s*TJ|T\*|Td|TD|'", bt.group(1), re.S):
                t = tok.group(0)
                if t.startswith(b"("):
                    line.append(_pdf_string(t[1:-1]))
                elif t in (b"T*", b"Td", b"TD", b"'") and line:
                    line.append("\n")
            texts.append("".join(line))
    return "\n".join(x.strip() for x in texts if x.strip())


def image(data: bytes, longest_edge: int) -> bytes:
    if data is None:
        return None
    from PIL import Image
    im = Image.open(io.BytesIO(data))
    w, h = im.size
    scale = min(1.0, float(longest_edge) / max(w, h))
    if scale < 1.0:
        im = im.resize((max(1, round(w * scale)), max(1, round(h * scale))))
    buf = io.BytesIO()
    im.save(buf, format="PNG")
    return buf.getvalue()


def call(name: str, args: list, n: int):
    def col(a):
        if isinstance(a, pa.Scalar):
            return [a.as_py()] * n
        return a.to_pylist()

    if name == "AI.PARSE_DOCUMENT":
        return pa.array([parse_document(x) for x in col(args[0])], pa.string())
    if name == "AI.IMAGE":
        edges = col(args[1])
        return pa.array([image(x, e) for x, e in zip(col(args[0]), edges)], pa.binary())
    if name == "AI.PDF_PAGES":
        from quail_b200.sql.pdf_render import DEFAULT_LONGEST_EDGE, pdf_pages
        pdfs = col(args[0])
        edges = col(args[1]) if len(args) > 1 else [DEFAULT_LONGEST_EDGE] * n
        firsts = col(args[2]) if len(args) > 2 else [1] * n
        lasts = col(args[3]) if len(args) > 3 else [None] * n
        out = [pdf_pages(d, int(e or DEFAULT_LONGEST_EDGE), int(f or 1), None if la is None else int(la))
               for d, e, f, la in zip(pdfs, edges, firsts, lasts)]
        return pa.array(out, PDF_PAGES_TYPE)
    from quail_b200.api.config import Refusal, RefusalError
    raise RefusalError(Refusal(reasons=(f"unknown document function {name}",), constraint="unsupported_function"))


PDF_PAGES_TYPE = pa.list_(pa.struct([("page", pa.int32()), ("image", pa.binary())]))
