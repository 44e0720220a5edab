"""AI.PDF_PAGES: each page of a PDF drawn as a PNG on the CPU, for a vision model to read.

A small PDF interpreter of this build's own, over PIL:
  - the file's objects are read by their `N G obj ... endobj` bodies, streams inflated
    (FlateDecode) where compressed; pages are found through the catalog's page tree (/Kids in
    order, /MediaBox inherited from parent nodes), or in object order when the tree is absent;
  - a page's content streams run through a graphics-state machine: q / Q, cm, the path
    operators (m l c v y h re, curves flattened to 8 segments) filled or stroked (f F f* S s
    B B* b b* n), the colour operators (g G rg RG k K), the text operators (BT ET Tf TL Td TD
    Tm T* Tj TJ ' ") drawn with the default FreeType face at the text matrix's size; images
    and other XObjects (Do) are drawn as light grey boxes, clipping is not applied;
  - the page is scaled so its longer side is `longest_edge` pixels at most and each side a
    multiple of 32 (one vision token per 32 x 32 pixels).
Fonts' own glyphs and encodings are not read: strings are shown as Latin-1 text. A page the
interpreter cannot draw gives None.

Reference: crates/quail-datafusion/src/functions/pdf_pages.rs (the same function with the hayro
renderer; the same arguments, size rule and result type list<struct<page int32, image binary>>).
"""

from __future__ import annotations

import io
import re
import zlib

SIDE_MULTIPLE = 32
DEFAULT_LONGEST_EDGE = 1536
MAX_LONGEST_EDGE = 8192

_OBJ = re.compile(rb"(\d+)\s+(\d+)\s+obj\b(.*?)\bendobj", re.S)
_REF = re.compile(rb"(\d+)\s+(\d+)\s+R\b")


def _objects(data: bytes) -> dict:
    return {int(m.group(1)): m.group(3) for m in _OBJ.finditer(data)}


def _dict_part(body: bytes) -> bytes:
    i = body.find(b"stream")
    return body if i < 0 else body[:i]


def _stream(body: bytes) -> bytes | None:
    m = re.search(rb"stream\r?\n", body)
    if m is None:
        return None
    end = body.rfind(b"endstream")
    raw = body[m.end():end if end > 0 else len(body)].rstrip(b"\r\n")
    if b"FlateDecode" in _dict_part(body):
        try:
            return zlib.decompress(raw)
        except zlib.error:
            try:
                return zlib.decompressobj().decompress(raw)
            except zlib.error:
                return None
    return raw


def _ref_of(dict_bytes: bytes, key: bytes):
    m = re.search(rb"/" + key + rb"\s+(\d+)\s+\d+\s+R", dict_bytes)
    return int(m.group(1)) if m else None


def _box(dict_bytes: bytes):
    m = re.search(rb"/MediaBox\s*\[([^\]]*)\]", dict_bytes)
    if not m:
        return None
    vals = [float(x) for x in re.findall(rb"-?\d*\.?\d+", m.group(1))]
    return vals if len(vals) == 4 else None


def pages_of(data: bytes) -> list[tuple[list, bytes]]:
    """[(media box, content bytes)] of each page, in order."""
    objs = _objects(data)
    is_page = {n for n, b in objs.items() if re.search(rb"/Type\s*/Page\b(?!s)", _dict_part(b))}
    order: list[int] = []
    root = _ref_of(data[data.rfind(b"trailer"):] if b"trailer" in data else b"", b"Root")
    if root is None:
        for n, b in objs.items():
            if re.search(rb"/Type\s*/Catalog", _dict_part(b)):
                root = n
                break
    parent_box: dict = {}

    def walk(n: int, box, depth: int = 0) -> None:
        if n not in objs or depth > 64:
            return
        d = _dict_part(objs[n])
        box = _box(d) or box
        if n in is_page:
            parent_box[n] = box
            order.append(n)
            return
        m = re.search(rb"/Kids\s*\[([^\]]*)\]", d)
        if m:
            for k in _REF.finditer(m.group(1)):
                walk(int(k.group(1)), box, depth + 1)
    if root is not None and root in objs:
        pages_ref = _ref_of(_dict_part(objs[root]), b"Pages")
        if pages_ref is not None:
            walk(pages_ref, None)
    if not order:
        order = sorted(is_page)
    out = []
    for n in order:
        d = _dict_part(objs[n])
        box = _box(d) or parent_box.get(n) or [0, 0, 612, 792]
        refs = []
        m = re.search(rb"/Contents\s*\[([^\]]*)\]", d)
        if m:
            refs = [int(k.group(1)) for k in _REF.finditer(m.group(1))]
        else:
            r = _ref_of(d, b"Contents")
            refs = [r] if r is not None else []
        content = b"\n".join(s for s in (_stream(objs[r]) if r in objs else None for r in refs) if s)
        out.append((box, content))
    return out


# ---------------------------------------------------------------- content streams
_TOKEN = re.compile(rb"""
    (?P<ws>\s+|%[^\r\n]*)
  | (?P<num>[+-]?(?:\d+\.?\d*|\.\d+))
  | (?P<name>/[^\s/\[\]()<>{}%]*)
  | (?P<str>\()
  | (?P<hex><[0-9A-Fa-f\s]*>)
  | (?P<dict><<|>>)
  | (?P<arr>[\[\]])
  | (?P<op>[A-Za-z'"*]+[0-9]?\*?|[{}])
""", re.X)


def _literal(data: bytes, i: int) -> tuple[bytes, int]:
    """The literal string starting after '(' at i: (bytes, index after ')')."""
    out, depth = bytearray(), 1
    esc = {ord("n"): 10, ord("r"): 13, ord("t"): 9, ord("b"): 8, ord("f"): 12}
    while i < len(data):
        c = data[i]
        if c == 0x5C and i + 1 < len(data):
            n = data[i + 1]
            if n in esc:
                out.append(esc[n])
                i += 2
            elif 0x30 <= n <= 0x37:
                j = i + 1
                while j < len(data) and j < i + 4 and 0x30 <= data[j] <= 0x37:
                    j += 1
                out.append(int(data[i + 1:j], 8) & 0xFF)
                i = j
            else:
                out.append(n)
                i += 2
            continue
        if c == 0x28:
            depth += 1
        elif c == 0x29:
            depth -= 1
            if depth == 0:
                return bytes(out), i + 1
        out.append(c)
        i += 1
    return bytes(out), i


def tokens(data: bytes):
    """Operands and operators of a content stream, in order: numbers as float, names as str
    ('/Name'), strings as bytes, arrays as lists, operators as ('op', name)."""
    stack: list[list] = [[]]
    i = 0
    while i < len(data):
        m = _TOKEN.match(data, i)
        if m is None:
            i += 1
            continue
        i = m.end()
        kind = m.lastgroup
        if kind == "ws" or kind == "dict":
            continue
        if kind == "num":
            stack[-1].append(float(m.group()))
        elif kind == "name":
            stack[-1].append(m.group().decode("latin-1"))
        elif kind == "str":
            s, i = _literal(data, i)
            stack[-1].append(s)
        elif kind == "hex":
            h = re.sub(rb"\s", b"", m.group()[1:-1])
            stack[-1].append(bytes.fromhex((h + b"0" if len(h) % 2 else h).decode()))
        elif kind == "arr":
            if m.group() == b"[":
                stack.append([])
            elif len(stack) > 1:
                arr = stack.pop()
                stack[-1].append(arr)
        else:
            yield ("op", m.group().decode("latin-1"), stack[-1])
            stack[-1] = []


def _mul(a, b):
    """3x2 affine matrices [a b c d e f]: a then b."""
    return [a[0] * b[0] + a[1] * b[2], a[0] * b[1] + a[1] * b[3], a[2] * b[0] + a[3] * b[2],
            a[2] * b[1] + a[3] * b[3], a[4] * b[0] + a[5] * b[2] + b[4], a[4] * b[1] + a[5] * b[3] + b[5]]


def _apply(m, x, y):
    return m[0] * x + m[2] * y + m[4], m[1] * x + m[3] * y + m[5]


def _rgb(vals, cmyk=False):
    if cmyk and len(vals) >= 4:
        c, m_, y, k = vals[:4]
        return tuple(int(255 * (1 - min(1.0, v + k))) for v in (c, m_, y))
    if len(vals) >= 3:
        return tuple(int(255 * max(0.0, min(1.0, v))) for v in vals[:3])
    g = int(255 * max(0.0, min(1.0, vals[0]))) if vals else 0
    return (g, g, g)


def _bezier(p0, p1, p2, p3, n=8):
    out = []
    for k in range(1, n + 1):
        t = k / n
        u = 1 - t
        out.append((u ** 3 * p0[0] + 3 * u * u * t * p1[0] + 3 * u * t * t * p2[0] + t ** 3 * p3[0],
                    u ** 3 * p0[1] + 3 * u * u * t * p1[1] + 3 * u * t * t * p2[1] + t ** 3 * p3[1]))
    return out


def page_size(box, longest_edge: int) -> tuple[int, int, float]:
    """(width, height, points-to-pixels scale) of a page drawn with its longer side at most
    `longest_edge` pixels, each side a whole number of 32-pixel blocks (at least one)."""
    w, h = abs(box[2] - box[0]), abs(box[3] - box[1])
    scale = longest_edge / max(w, h, 1e-6)
    W = max(SIDE_MULTIPLE, int(w * scale) // SIDE_MULTIPLE * SIDE_MULTIPLE)
    H = max(SIDE_MULTIPLE, int(h * scale) // SIDE_MULTIPLE * SIDE_MULTIPLE)
    return W, H, scale


def render_page(box, content: bytes, longest_edge: int = DEFAULT_LONGEST_EDGE) -> bytes:
    """One page's content stream drawn as PNG bytes."""
    from PIL import Image, ImageDraw, ImageFont
    W, H, scale = page_size(box, longest_edge)
    sx, sy = W / max(abs(box[2] - box[0]), 1e-6), H / max(abs(box[3] - box[1]), 1e-6)
    # device matrix: PDF user space (origin bottom-left, points) -> pixels (origin top-left)
    dev = [sx, 0.0, 0.0, -sy, -box[0] * sx, box[3] * sy]
    img = Image.new("RGB", (W, H), (255, 255, 255))
    draw = ImageDraw.Draw(img)
    gs = {"ctm": [1.0, 0, 0, 1.0, 0, 0], "fill": (0, 0, 0), "stroke": (0, 0, 0), "lw": 1.0}
    stack: list = []
    path: list[list] = []
    cur = None
    tm = tlm = [1.0, 0, 0, 1.0, 0, 0]
    font_size, leading = 12.0, 0.0
    fonts: dict = {}

    def to_px(x, y):
        return _apply(_mul(gs["ctm"], dev), x, y)

    def paint(fill: bool, stroke: bool):
        for sub in path:
            pts = [to_px(*p) for p in sub]
            if len(pts) >= 3 and fill:
                draw.polygon(pts, fill=gs["fill"])
            if len(pts) >= 2 and stroke:
                width = max(1, int(round(gs["lw"] * abs(gs["ctm"][0]) * sx)))
                draw.line(pts, fill=gs["stroke"], width=width)

    def show(text: bytes):
        nonlocal tm
        m = _mul(_mul(tm, gs["ctm"]), dev)
        size_px = max(1, int(round(font_size * (m[2] ** 2 + m[3] ** 2) ** 0.5)))
        font = fonts.get(size_px)
        if font is None:
            font = fonts[size_px] = ImageFont.load_default(size=min(size_px, 512))
        s = text.decode("latin-1")
        x, y = _apply(m, 0, 0)
        draw.text((x, y - size_px * 0.8), s, fill=gs["fill"], font=font)
        adv = font.getlength(s) / max((m[0] ** 2 + m[1] ** 2) ** 0.5, 1e-6)
        tm = _mul([1, 0, 0, 1, adv, 0], tm)

    for _, op, a in tokens(content):
        try:
            if op == "q":
                stack.append(dict(gs))
            elif op == "Q":
                if stack:
                    gs = stack.pop()
            elif op == "cm" and len(a) >= 6:
                gs["ctm"] = _mul([float(v) for v in a[:6]], gs["ctm"])
            elif op == "w" and a:
                gs["lw"] = float(a[0])
            elif op in ("g", "rg", "k"):
                gs["fill"] = _rgb([float(v) for v in a if isinstance(v, float)], op == "k")
            elif op in ("G", "RG", "K"):
                gs["stroke"] = _rgb([float(v) for v in a if isinstance(v, float)], op == "K")
            elif op == "m" and len(a) >= 2:
                cur = (a[0], a[1])
                path.append([cur])
            elif op == "l" and len(a) >= 2 and path:
                cur = (a[0], a[1])
                path[-1].append(cur)
            elif op in ("c", "v", "y") and path and cur is not None:
                if op == "c" and len(a) >= 6:
                    pts = _bezier(cur, (a[0], a[1]), (a[2], a[3]), (a[4], a[5]))
                elif op == "v" and len(a) >= 4:
                    pts = _bezier(cur, cur, (a[0], a[1]), (a[2], a[3]))
                elif op == "y" and len(a) >= 4:
                    pts = _bezier(cur, (a[0], a[1]), (a[2], a[3]), (a[2], a[3]))
                else:
                    continue
                path[-1].extend(pts)
                cur = pts[-1]
            elif op == "h" and path and path[-1]:
                path[-1].append(path[-1][0])
            elif op == "re" and len(a) >= 4:
                x, y, w, h = a[:4]
                path.append([(x, y), (x + w, y), (x + w, y + h), (x, y + h), (x, y)])
                cur = (x, y)
            elif op in ("f", "F", "f*"):
                paint(True, False)
                path, cur = [], None
            elif op in ("S", "s"):
                paint(False, True)
                path, cur = [], None
            elif op in ("B", "B*", "b", "b*"):
                paint(True, True)
                path, cur = [], None
            elif op == "n":
                path, cur = [], None
            elif op == "BT":
                tm = tlm = [1.0, 0, 0, 1.0, 0, 0]
            elif op == "Tf" and len(a) >= 2:
                font_size = float(a[1])
            elif op == "TL" and a:
                leading = float(a[0])
            elif op in ("Td", "TD") and len(a) >= 2:
                if op == "TD":
                    leading = -float(a[1])
                tlm = _mul([1, 0, 0, 1, float(a[0]), float(a[1])], tlm)
                tm = tlm
            elif op == "Tm" and len(a) >= 6:
                tm = tlm = [float(v) for v in a[:6]]
            elif op == "T*":
                tlm = _mul([1, 0, 0, 1, 0, -leading], tlm)
                tm = tlm
            elif op == "Tj" and a and isinstance(a[0], bytes):
                show(a[0])
            elif op == "TJ" and a and isinstance(a[0], list):
                for part in a[0]:
                    if isinstance(part, bytes):
                        show(part)
                    elif isinstance(part, float):
                        tm = _mul([1, 0, 0, 1, -part / 1000.0 * font_size, 0], tm)
            elif op in ("'", '"') and a and isinstance(a[-1], bytes):
                tlm = _mul([1, 0, 0, 1, 0, -leading], tlm)
                tm = tlm
                show(a[-1])
            elif op == "Do":
                # an image or form XObject: its unit square, drawn as a light box
                pts = [to_px(*p) for p in ((0, 0), (1, 0), (1, 1), (0, 1))]
                draw.polygon(pts, fill=(225, 225, 225))
        except (TypeError, ValueError, ZeroDivisionError, OverflowError):
            continue
    buf = io.BytesIO()
    img.save(buf, format="PNG")
    return buf.getvalue()


def pdf_pages(data: bytes, longest_edge: int = DEFAULT_LONGEST_EDGE, first: int = 1, last: int | None = None):
    """[{"page": n, "image": PNG bytes or None}] for pages first..last (numbered from 1)."""
    if data is None:
        return None
    if not 1 <= longest_edge <= MAX_LONGEST_EDGE:
        raise ValueError(f"longest_edge must be in [1, {MAX_LONGEST_EDGE}], not {longest_edge}")
    pages = pages_of(bytes(data))
    last = len(pages) if last is None else min(last, len(pages))
    out = []
    for n in range(max(1, first), last + 1):
        box, content = pages[n - 1]
        try:
            png = render_page(box, content, longest_edge)
        except Exception:  # noqa: BLE001 - a page the interpreter cannot draw reads as None
            png = None
        out.append({"page": n, "image": png})
    return out
