"""An extraction tested with LIKE reads only the documents that hold the pattern's text.

AI.EXTRACT copies its answers from the document, so `answer['f'] LIKE '%2027%'`
can only pass on documents that contain '2027': the executor drops the others
before asking the model (case-insensitively, on the pattern's longest word).
The rows are the same as with the demand rules off; fewer questions are asked.
Reference: crates/quail-datafusion/src/rules/substring.rs.
"""

import zlib

import numpy as np
import pyarrow as pa

import quail_b200 as quail
from oracle import OracleEngine


class CopyingOracle(OracleEngine):
    """Extraction answers copied from the document: one of its words, by hash."""

    def answer(self, call, doc):
        if call.kind == "extract":
            words = str(doc).split()
            return words[zlib.crc32((call.tail + str(doc)).encode()) % len(words)]
        return super().answer(call, doc)


def _table(n=80, seed=5):
    rng = np.random.default_rng(seed)
    words = ["lease", "ends", "2026", "2027", "2028", "rent", "renewal", "tenant"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(2, 6)))) for _ in range(n)]
    return pa.table({"id": list(range(n)), "body": bodies})


def _run(sql, pushdown=True):
    oracle = CopyingOracle()
    s = quail.Session(config=quail.EngineConfig(model="qwen3-tiny", device="cpu"))
    s.register("leases", quail.DocumentProvider.from_table(_table(), id_col="id"))
    s.attach_engine(oracle)
    if not pushdown:
        s.sql("SET quail.pushdown = false").run()
    return s.sql(sql).collect().to_pylist(), len(oracle.asked)


def test_extraction_like_reads_only_documents_with_the_text():
    sql = ("SELECT id FROM leases WHERE AI.EXTRACT(body, {'end': 'When does the lease end?'})['end'] "
           "LIKE '%2027%' ORDER BY id")
    rows, asked = _run(sql)
    rows_off, asked_off = _run(sql, pushdown=False)
    assert rows == rows_off and rows
    bodies = set(_table().column("body").to_pylist())          # one question per distinct document
    assert asked == sum("2027" in b for b in bodies) < asked_off == len(bodies)


def test_negated_and_wildcard_only_patterns_read_every_document():
    for cond in ("NOT LIKE '%2027%'", "LIKE '%'"):
        sql = f"SELECT id FROM leases WHERE AI.EXTRACT(body, {{'end': 'When?'}})['end'] {cond} ORDER BY id"
        rows, asked = _run(sql)
        rows_off, asked_off = _run(sql, pushdown=False)
        assert rows == rows_off
        assert asked == asked_off == len(set(_table().column("body").to_pylist()))
