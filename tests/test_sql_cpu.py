"""SQL semantics of the executor without a model: every query against a plain
Python statement of the same result over the same small tables."""

import math

import pyarrow as pa
import pytest

import quail_b200 as quail

T = {"id": [1, 2, 3, 4, 5, 6], "g": ["a", "b", "a", "c", "b", "a"], "x": [10, 20, None, 40, 50, 60],
     "s": ["Foo", "bar", "Baz", "qux", "Quux", "foo"]}
U = {"g": ["a", "b", "d"], "label": ["A", "B", "D"]}
ROWS = [dict(zip(T, v)) for v in zip(*T.values())]


@pytest.fixture(scope="module")
def s():
    sess = quail.Session(config=quail.EngineConfig(model="qwen3-tiny", device="cpu"))
    sess.register("t", pa.table(T))
    sess.register("u", pa.table(U))
    yield sess
    sess.close()


def col(s, q, name=None):
    t = s.sql(q).collect()
    return t.column(name or t.column_names[0]).to_pylist()


def ids(pred):
    return [r["id"] for r in ROWS if pred(r)]


@pytest.mark.parametrize("where,pred", [
    ("x > 15 AND g = 'a'", lambda r: r["x"] is not None and r["x"] > 15 and r["g"] == "a"),
    ("x > 15 OR g = 'c'", lambda r: (r["x"] is not None and r["x"] > 15) or r["g"] == "c"),
    ("NOT (g = 'a')", lambda r: r["g"] != "a"),
    ("g IN ('a', 'c')", lambda r: r["g"] in ("a", "c")),
    ("g NOT IN ('a', 'c')", lambda r: r["g"] not in ("a", "c")),
    ("x BETWEEN 20 AND 50", lambda r: r["x"] is not None and 20 <= r["x"] <= 50),
    ("s LIKE 'f%'", lambda r: r["s"].startswith("f")),
    ("s ILIKE 'f%'", lambda r: r["s"].lower().startswith("f")),
    ("x IS NULL", lambda r: r["x"] is None),
    ("x IS NOT NULL", lambda r: r["x"] is not None),
    ("REGEXP_LIKE(s, '^[Ff]')", lambda r: r["s"][0] in "Ff"),
    ("g IN (SELECT g FROM u)", lambda r: r["g"] in U["g"]),
    ("x > (SELECT AVG(x) FROM t)", lambda r: r["x"] is not None and r["x"] > 36),
])
def test_where(s, where, pred):
    assert sorted(col(s, f"SELECT id FROM t WHERE {where}")) == ids(pred)


def test_projection_and_case(s):
    assert col(s, "SELECT x * 2 + 1 AS y FROM t ORDER BY id") == [None if r["x"] is None else r["x"] * 2 + 1
                                                                   for r in ROWS]
    want = ["small" if r["x"] is None or r["x"] <= 15 else "mid" if r["x"] <= 30 else "big" for r in ROWS]
    q = "SELECT CASE WHEN x > 30 THEN 'big' WHEN x > 15 THEN 'mid' ELSE 'small' END AS c FROM t ORDER BY id"
    assert col(s, q) == want
    assert col(s, "SELECT COALESCE(x, 0) AS v FROM t ORDER BY id") == [r["x"] or 0 for r in ROWS]
    assert col(s, "SELECT LOWER(s) AS v FROM t ORDER BY id") == [r["s"].lower() for r in ROWS]
    assert col(s, "SELECT s || '-' || g AS v FROM t ORDER BY id") == [f"{r['s']}-{r['g']}" for r in ROWS]
    assert col(s, "SELECT SUBSTR(s, 1, 2) AS v FROM t ORDER BY id") == [r["s"][:2] for r in ROWS]


def test_group_by_aggregates_and_having(s):
    t = s.sql("SELECT g, COUNT(*) AS n, SUM(x) AS sx, MIN(x) AS mn, MAX(x) AS mx FROM t GROUP BY g ORDER BY g")
    got = t.collect().to_pylist()
    for row in got:
        xs = [r["x"] for r in ROWS if r["g"] == row["g"] and r["x"] is not None]
        assert row["n"] == sum(1 for r in ROWS if r["g"] == row["g"])
        assert row["sx"] == sum(xs) and row["mn"] == min(xs) and row["mx"] == max(xs)
    assert [r["g"] for r in got] == ["a", "b", "c"]
    assert sorted(col(s, "SELECT g FROM t GROUP BY g HAVING COUNT(*) > 1")) == ["a", "b"]
    assert col(s, "SELECT COUNT(DISTINCT g) AS n FROM t") == [3]
    avg = col(s, "SELECT AVG(x) AS a FROM t")[0]
    assert math.isclose(avg, sum(r["x"] for r in ROWS if r["x"] is not None) / 5)


def test_order_limit_offset_distinct_union(s):
    assert col(s, "SELECT id FROM t ORDER BY g DESC, id ASC") == [4, 2, 5, 1, 3, 6]
    assert col(s, "SELECT id FROM t ORDER BY id LIMIT 2 OFFSET 2") == [3, 4]
    assert sorted(col(s, "SELECT DISTINCT g FROM t")) == ["a", "b", "c"]
    assert len(col(s, "SELECT id FROM t UNION ALL SELECT id FROM t")) == 12
    assert col(s, "WITH big AS (SELECT * FROM t WHERE x > 15) SELECT id FROM big ORDER BY id") == [2, 4, 5, 6]


def test_joins(s):
    inner = s.sql("SELECT t.id, u.label FROM t JOIN u ON t.g = u.g ORDER BY t.id").collect().to_pylist()
    assert [(r["id"], r["label"]) for r in inner] == [(1, "A"), (2, "B"), (3, "A"), (5, "B"), (6, "A")]
    left = s.sql("SELECT t.id, u.label FROM t LEFT JOIN u ON t.g = u.g ORDER BY t.id").collect().to_pylist()
    assert [r["label"] for r in left] == ["A", "B", "A", None, "B", "A"]
    cross = col(s, "SELECT t1.id FROM t t1 CROSS JOIN u t2 WHERE t1.g = t2.g ORDER BY t1.id")
    assert cross == [1, 2, 3, 5, 6]


def test_errors_are_query_errors(s):
    with pytest.raises(Exception):
        s.sql("SELEC id FROM t").collect()
    with pytest.raises(Exception):
        s.sql("SELECT nope FROM t").collect()
    with pytest.raises(Exception):
        s.sql("SELECT id FROM missing").collect()
