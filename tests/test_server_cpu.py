"""Quail Server on CPU: Flight calls, the persistent queue, tokens, and a remote Session."""

import json
import os

import numpy as np
import pyarrow as pa
import pyarrow.flight as flight
import pytest

import quail_b200 as quail
from quail_b200.server.client import QueryFailedError, ServerClient
from quail_b200.server.queue import STOPPED
from quail_b200.server.service import QuailFlightServer

Q = "SELECT r.id FROM reviews r WHERE AI.IF(PROMPT('Does the review discuss the ending? {0}', r.body))"


def _table(n=16, seed=0):
    rng = np.random.default_rng(seed)
    words = ["ending", "music", "cast", "plot", "money", "great", "bad", "long", "short", "story"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 10)))) for _ in range(n)]
    return pa.table({"id": list(range(n)), "body": bodies})


@pytest.fixture(scope="module")
def session():
    cfg = quail.EngineConfig(model="qwen3-tiny", device="cpu", chunk_tokens=256)
    with quail.Session(config=cfg) as s:
        yield s


@pytest.fixture()
def server(session, tmp_path):
    srv = QuailFlightServer(session, str(tmp_path / "data"), token="")
    yield srv
    srv.shutdown()


def test_submit_wait_rows_match_local(session, server):
    c = ServerClient(server.endpoint, token="")
    c.upload("reviews", _table(), "id")
    st = c.submit(Q, query_id="q1")
    assert st.id == "q1" and st.state in ("queued", "running", "succeeded")
    again = c.submit(Q, query_id="q1")      # the same id runs once
    assert again.submitted_at == st.submitted_at
    from quail_b200.server.client import QueryRun
    run = QueryRun(c, "q1")
    final = run.wait(wait_s=0.5)
    assert final.state == "succeeded", final
    got = run.result().table.column("id").to_pylist()
    session.register("reviews", quail.DocumentProvider.from_table(_table(), id_col="id"))
    want = session.sql(Q).collect().column("id").to_pylist()
    assert got == want
    assert final.num_rows == len(want) and final.plans
    assert c.report("q1")[0]["evaluated_documents"] == 16
    assert c.answers("q1")["next"] >= 1
    assert [s.id for s in c.submissions()] == ["q1"]
    assert "AI" in c.explain(Q) or len(c.explain(Q)) > 0
    # a direct SQL ticket runs at once
    assert c.sql("SELECT id FROM reviews WHERE id < 3").column("id").to_pylist() == [0, 1, 2]
    c.close()


def test_cancel_and_failures(server):
    c = ServerClient(server.endpoint, token="")
    c.upload("reviews", _table(), "id")
    # a long query occupies the runner; the next one is cancelled while queued
    long_q = "SELECT r.id FROM reviews r WHERE AI.IF(PROMPT('Is it about money? {0}', r.body))"
    a = c.submit(long_q, query_id="a")
    b = c.submit(Q, query_id="b")
    st = c.cancel("b")
    assert st.state in ("cancelled", "running", "succeeded")
    from quail_b200.server.client import QueryRun
    assert QueryRun(c, "a").wait(0.5).state == "succeeded"
    final_b = QueryRun(c, "b").wait(0.5)
    if st.state == "cancelled":
        assert final_b.state == "cancelled"
        with pytest.raises(QueryFailedError):
            QueryRun(c, "b").result()
    bad = c.submit("SELECT nope FROM missing_table", query_id="bad")
    assert QueryRun(c, bad.id).wait(0.5).state == "failed"
    with pytest.raises(flight.FlightError):
        c.status("unknown-id")
    # status_after answers at once when a newer revision exists
    s0 = c.status("a", after=0, wait_s=5)
    assert s0.revision > 0
    del a
    c.close()


def test_restart_keeps_submissions(session, tmp_path):
    d = str(tmp_path / "data")
    srv = QuailFlightServer(session, d, token="")
    c = ServerClient(srv.endpoint, token="")
    c.upload("reviews", _table(), "id")
    c.submit(Q, query_id="done")
    from quail_b200.server.client import QueryRun
    assert QueryRun(c, "done").wait(0.5).state == "succeeded"
    rows = QueryRun(c, "done").result().table
    c.close()
    srv.shutdown()
    # a submission an earlier server left running is marked failed on reopen
    os.makedirs(os.path.join(d, "halfway"))
    with open(os.path.join(d, "halfway", "status.json"), "w") as f:
        json.dump({"id": "halfway", "sql": Q, "state": "running", "submitted_at": 1.0, "revision": 3}, f)
    srv2 = QuailFlightServer(session, d, token="")
    c2 = ServerClient(srv2.endpoint, token="")
    ids = {s.id: s for s in c2.submissions()}
    assert ids["done"].state == "succeeded"
    assert ids["halfway"].state == "failed" and ids["halfway"].error == STOPPED
    assert QueryRun(c2, "done").result().table.equals(rows)
    c2.close()
    srv2.shutdown()


def test_bearer_token(session, tmp_path):
    srv = QuailFlightServer(session, str(tmp_path / "data"), token="s3cret")
    try:
        with pytest.raises(flight.FlightUnauthenticatedError):
            ServerClient(srv.endpoint, token="").submissions()
        with pytest.raises(flight.FlightUnauthenticatedError):
            ServerClient(srv.endpoint, token="wrong").submissions()
        assert ServerClient(srv.endpoint, token="s3cret").submissions() == []
    finally:
        srv.shutdown()


def test_remote_session(server):
    with quail.Session(endpoint=server.endpoint, token="") as rs:
        rs.register("reviews", quail.DocumentProvider.from_table(_table(), id_col="id"))
        q = rs.sql(Q)
        got = q.collect().column("id").to_pylist()
        run = q.submit(query_id="again")
        assert run.wait(0.5).state == "succeeded"
        assert rs.get_run("again").result().table.column("id").to_pylist() == got
        streamed = rs.sql(Q).execute_stream(batch_rows=4).read_all()
        assert streamed.column("id").to_pylist() == got
        with pytest.raises(RuntimeError):
            q.plan()


def test_timeout_stops_the_run(server):
    import time
    c = ServerClient(server.endpoint, token="")
    c.upload("reviews", _table(64, seed=3), "id")
    st = c.submit(Q, query_id="slow", timeout_s=0.05)
    from quail_b200.server.client import QueryRun
    t0 = time.time()
    final = QueryRun(c, st.id).wait(0.5)
    if final.state == "failed":
        assert "timed out" in final.error
    else:  # the tiny model may finish within the limit on a fast host
        assert final.state == "succeeded" and time.time() - t0 < 5
    c.close()
