"""Plan snapshots: the explain text of representative queries must equal the stored text.

A change to planning shows up as a diff of these files; regenerate them with
QUAIL_UPDATE_SNAPSHOTS=1 after checking that the new plans are right (the
reference's tests/bench/test_plan_snapshots.py does the same over its
benchmark queries).
"""

import os
import pathlib

import pyarrow as pa
import pytest

import quail_b200 as quail

HERE = pathlib.Path(__file__).parent / "fixtures" / "plan_snapshots"

QUERIES = {
    "filter_then_score": "SELECT id, AI.SCORE(PROMPT('Is the review positive? {0}', body)) AS s FROM reviews "
                         "WHERE stars > 2 AND AI.IF(PROMPT('Does it mention the plot? {0}', body)) "
                         "ORDER BY s DESC LIMIT 5",
    "classify": "SELECT id, AI.CLASSIFY(body, ['praise', 'complaint', 'question']) AS k FROM reviews",
    "map_and_extract": "SELECT id, AI.MAP(body, 'Summarize in five words.', 16) AS m, "
                       "AI.EXTRACT(body, ['Which actor?']) AS e FROM reviews WHERE stars = 5",
    "two_filters": "SELECT id FROM reviews WHERE AI.IF(PROMPT('Is it long? {0}', body)) "
                   "AND AI.IF(PROMPT('Is it funny? {0}', body))",
    "join": "SELECT r.id, m.title FROM reviews r JOIN movies m ON r.movie = m.id "
            "WHERE AI.IF(PROMPT('Is {0} about a sequel?', r.body))",
    "aggregate": "SELECT stars, COUNT(*) AS n FROM reviews WHERE AI.IF(PROMPT('Is it sarcastic? {0}', body)) "
                 "GROUP BY stars ORDER BY stars",
    "selectivity": "SELECT id, AI.SCORE(PROMPT('Is it positive? {0}', body)) AS s FROM reviews "
                   "WHERE AI.IF(PROMPT('Is it about acting? {0}', body), {'selectivity': 0.25})",
    "ai_join_anchor": "SELECT r.id, m.title FROM reviews r JOIN movies m "
                      "ON AI.IF(PROMPT('Is {0} a review of the film {1}?', r.body, m.title))",
    "cost_order": "SELECT id FROM reviews WHERE AI.IF(PROMPT('Is this a long and detailed review that discusses "
                  "the acting, the music and the plot of the film at length? {0}', body), {'selectivity': 0.5}) "
                  "AND AI.IF(PROMPT('Is it funny? {0}', body), {'selectivity': 0.5})",
    "cte": "WITH good AS (SELECT id, body FROM reviews WHERE stars >= 4) "
           "SELECT id, AI.SCORE(PROMPT('Would they rewatch? {0}', body)) AS s FROM good",
}


@pytest.fixture(scope="module")
def session():
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=256)
    reviews = pa.table({"id": list(range(8)), "movie": [0, 1, 0, 2, 1, 0, 2, 1], "stars": [1, 5, 3, 4, 2, 5, 4, 3],
                        "body": [f"review number {i} of a film" for i in range(8)]})
    movies = pa.table({"id": [0, 1, 2], "title": ["A", "B", "C"]})
    with quail.Session(config=cfg) as s:
        s.register("reviews", reviews)
        s.register("movies", movies)
        yield s


@pytest.mark.parametrize("name", sorted(QUERIES))
def test_plan_snapshot(session, name):
    text = session.sql(QUERIES[name]).explain().rstrip() + "\n"
    path = HERE / f"{name}.txt"
    if os.environ.get("QUAIL_UPDATE_SNAPSHOTS") == "1":
        path.write_text(text)
    assert path.exists(), f"no snapshot for {name}; run with QUAIL_UPDATE_SNAPSHOTS=1"
    assert text == path.read_text(), f"plan of {name} changed:\n{text}"
