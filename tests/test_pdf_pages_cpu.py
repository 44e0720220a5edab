"""AI.PDF_PAGES: PDF pages drawn on the CPU, unnested into rows, read by a vision model."""

import io
import zlib

import numpy as np
import pyarrow as pa
import pytest
from PIL import Image

import quail_b200 as quail
from quail_b200.sql.pdf_render import page_size, pages_of, pdf_pages


def _pdf() -> bytes:
    one = b"BT /F1 24 Tf 72 700 Td (Invoice 42) Tj 0 -30 Td (Total due) Tj ET 0 0 1 rg 100 100 200 50 re f"
    two = zlib.compress(b"q 2 0 0 2 0 0 cm 1 0 0 RG 10 10 m 100 100 l S Q BT /F1 18 Tf 50 50 Td (Page two) Tj ET")
    parts = [b"%PDF-1.4\n1 0 obj << /Type /Catalog /Pages 2 0 R >> endobj\n",
             b"2 0 obj << /Type /Pages /Kids [5 0 R 3 0 R] /Count 2 /MediaBox [0 0 612 792] >> endobj\n",
             b"3 0 obj << /Type /Page /Parent 2 0 R /Contents 4 0 R >> endobj\n",
             b"4 0 obj << /Length " + str(len(one)).encode() + b" >> stream\n" + one + b"\nendstream endobj\n",
             b"5 0 obj << /Type /Page /Parent 2 0 R /MediaBox [0 0 300 300] /Contents 6 0 R >> endobj\n",
             b"6 0 obj << /Length " + str(len(two)).encode() + b" /Filter /FlateDecode >> stream\n" + two
             + b"\nendstream endobj\n", b"trailer << /Root 1 0 R >>\n%%EOF"]
    return b"".join(parts)


def test_pages_follow_the_page_tree_and_inherit_the_media_box():
    pages = pages_of(_pdf())
    assert [box for box, _ in pages] == [[0, 0, 300, 300], [0, 0, 612, 792]]   # /Kids order: 5, then 3
    assert b"Page two" in pages[0][1]                                             # inflated


def test_drawing():
    out = pdf_pages(_pdf(), 256)
    assert [p["page"] for p in out] == [1, 2]
    a = np.asarray(Image.open(io.BytesIO(out[1]["image"])))
    assert a.shape[0] % 32 == 0 and a.shape[1] % 32 == 0 and max(a.shape[:2]) <= 256
    W, H, scale = page_size([0, 0, 612, 792], 256)
    # the blue rectangle (100..300 x 100..150 points, origin bottom-left)
    y, x = int(H - 125 * H / 792), int(200 * W / 612)
    assert tuple(a[y, x]) == (0, 0, 255)
    # text draws dark pixels near the top left
    assert (a[: H // 3, : W // 2] < 100).all(axis=2).any()
    # the stroked red line of page one (scaled by its cm)
    b = np.asarray(Image.open(io.BytesIO(out[0]["image"])))
    assert ((b[..., 0] > 200) & (b[..., 1] < 80)).any()
    assert [p["page"] for p in pdf_pages(_pdf(), 128, 2, 2)] == [2]
    with pytest.raises(ValueError, match="longest_edge"):
        pdf_pages(_pdf(), 0)


def test_sql_pages_into_rows_and_a_vision_model():
    t = pa.table({"id": [7], "pdf": pa.array([_pdf()], pa.binary())})
    cfg = quail.EngineConfig(model="qwen3.5-vl-tiny", device="cpu", extra={"image_longest": 128})
    with quail.Session(config=cfg) as s:
        s.register("docs", quail.DocumentProvider.from_table(t, id_col="id"))
        pages = s.sql("SELECT p.id, p.u['page'] AS page, p.u['image'] AS image FROM "
                      "(SELECT d.id, UNNEST(AI_PDF_PAGES(d.pdf, 128)) AS u FROM docs d) p").collect()
        assert pages.column("page").to_pylist() == [1, 2] and pages.column("id").to_pylist() == [7, 7]
        s.register("pages", quail.DocumentProvider.from_table(pages.append_column("k", pa.array([0, 1])),
                                                              id_col="k"))
        got = s.sql("SELECT page, AI.SCORE(PROMPT('Is {0} an invoice?', image)) AS p FROM pages").collect()
        assert all(0 < p < 1 for p in got.column("p").to_pylist())
