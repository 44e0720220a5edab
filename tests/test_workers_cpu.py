"""Data-parallel workers on the host: each question asked once, same rows as one replica,
and failures (a worker that raises, exits mid-region, or never connects) handled on the host.

Workers here run the fp32 tiny model on CPU; nothing touches a GPU.
"""

import os

import numpy as np
import pyarrow as pa
import pytest

import quail_b200 as quail
from quail_b200 import _native
from quail_b200.api.engine import CallSpec
from quail_b200.api.prompts import bind_prompt
from quail_b200.runtime.workers import WorkerError, WorkerPool

pytestmark = pytest.mark.slow


def _table(n=20):
    rng = np.random.default_rng(5)
    words = ["alpha", "beta", "gamma", "delta", "omega"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(2, 8)))) for _ in range(n)]
    bodies[3] = bodies[7]  # a repeated document is read once
    return pa.table({"id": list(range(n)), "body": bodies})


def _cfg(gpus):
    return quail.EngineConfig(model="qwen3-tiny", device="cpu", gpus=gpus, chunk_tokens=256)


QUERY = "SELECT id, AI.SCORE(PROMPT('Is it greek? {0}', body)) AS s FROM t WHERE AI.IF(PROMPT('Short? {0}', body)) ORDER BY id"


def test_two_workers_return_the_rows_of_one_and_ask_each_question_once():
    t = _table()
    with quail.Session(config=_cfg(1)) as one:
        one.register("t", t)
        want = one.sql(QUERY).collect()
    with quail.Session(config=_cfg(2)) as two:
        two.register("t", t)
        res = two.sql(QUERY).run()
        got = res.table
        per = res.report["regions"][0]["per_worker"]
    assert got.column("id").to_pylist() == want.column("id").to_pylist()
    assert np.allclose(got.column("s").to_pylist(), want.column("s").to_pylist(), atol=1e-5)
    # 19 distinct documents, each filtered once, across both workers
    assert sum(p["documents"] for p in per) == 19
    assert all(p["documents"] > 0 for p in per)


def _region(pool):
    bp = bind_prompt("Short? {0}")
    return pool.run_region(bp.preamble, _table().column("body").to_pylist(),
                           [CallSpec(kind="filter", tail=bp.tail, name="f")])


def test_a_worker_that_raises_fails_the_region_with_its_traceback(monkeypatch):
    monkeypatch.setenv("QB_FAULT", "raise:1")
    pool = WorkerPool(_cfg(2))
    try:
        with pytest.raises(WorkerError, match="injected failure in worker 1"):
            _region(pool)
        assert pool.alive()  # the worker reported the error and keeps serving
    finally:
        pool.close()


def test_a_worker_that_exits_mid_region_fails_it_and_the_next_region_revives():
    os.environ["QB_FAULT"] = "exit:0"
    try:
        pool = WorkerPool(_cfg(2))
    finally:
        os.environ.pop("QB_FAULT")
    try:
        with pytest.raises(WorkerError, match="worker 0"):
            _region(pool)
        assert not pool.alive()
        # the children were spawned with the fault; revive re-spawns without it
        out = _region(pool)
        assert len(out.values) == 20
    finally:
        pool.close()


def test_a_worker_that_never_connects_is_an_error(monkeypatch):
    monkeypatch.setenv("QB_FAULT", "noconnect:1")
    with pytest.raises(WorkerError, match="exited"):
        WorkerPool(_cfg(2))


def test_an_oversized_frame_is_refused_before_allocation():
    import threading
    path = f"/tmp/qb-frame-{os.getpid()}.sock"
    lfd = _native.listen_unix(path)

    def peer():
        fd = _native.connect_unix(path, 2000)
        _native.send_frame(fd, b"x" * 1000, 2000)

    th = threading.Thread(target=peer)
    th.start()
    fd = _native.accept_unix(lfd, 2000)
    with pytest.raises(_native.IpcError, match="exceeds the limit"):
        _native.recv_frame(fd, 100, 2000)
    th.join()
    _native.close_fd(fd)
    _native.close_fd(lfd)
    os.unlink(path)


def _many(n=40):
    rng = np.random.default_rng(9)
    words = ["alpha", "beta", "gamma", "delta", "omega", "sigma", "kappa"]
    return [" ".join(rng.choice(words, size=int(rng.integers(20, 60)))) for _ in range(n)]


def test_workers_stream_answers_over_the_ask_channel():
    bp = bind_prompt("Short? {0}")
    docs = _many()
    got = {}

    def on_rows(rows, values):
        for r in rows:
            assert r not in got          # each row arrives once
            got[r] = values
    pool = WorkerPool(_cfg(2))
    try:
        out = pool.run_region(bp.preamble, docs, [CallSpec(kind="filter", tail=bp.tail, name="f")], on_rows=on_rows)
    finally:
        pool.close()
    assert sorted(got) == list(range(len(docs)))
    assert all(got[r] == out.values[r] for r in got)


def test_a_stop_answer_ends_the_region_with_the_rows_finished_so_far():
    bp = bind_prompt("Short? {0}")
    docs = _many()
    asked, seen = [], []

    def stop():
        # the fetch demand of a LIMIT: enough rows came back, stop asking
        asked.append(1)
        return len(seen) >= 5
    pool = WorkerPool(quail.EngineConfig(model="qwen3-tiny", device="cpu", gpus=2, chunk_tokens=128))
    pool.ask_every_s = 0.0               # ask between every two passes
    try:
        full = pool.run_region(bp.preamble, docs, [CallSpec(kind="filter", tail=bp.tail, name="f")])
        part = pool.run_region(bp.preamble, docs, [CallSpec(kind="filter", tail=bp.tail, name="f")], stop=stop,
                               on_rows=lambda rows, v: seen.extend(rows))
    finally:
        pool.close()
    assert asked
    done = [i for i, v in enumerate(part.values) if v]
    assert 0 < len(done) < len(docs)
    assert all(part.values[i] == full.values[i] for i in done)
    assert part.stats["asked"] < full.stats["asked"]


def test_interrupt_fails_regions_until_resume():
    pool = WorkerPool(_cfg(2))
    try:
        _region(pool)
        pool.interrupt()
        with pytest.raises(WorkerError, match="interrupted"):
            _region(pool)
        pool.resume()
        out = _region(pool)                # the workers are revived and the models reloaded
        assert len(out.values) == 20
    finally:
        pool.close()


def test_session_interrupt_and_resume_on_one_engine():
    from quail_b200.engine.stage_executor import QueryCancelled
    with quail.Session(config=_cfg(1)) as s:
        s.register("t", _table())
        s.sql(QUERY).collect()
        s.interrupt()
        with pytest.raises(QueryCancelled):
            s.sql(QUERY).collect()
        s.resume()
        assert s.sql(QUERY).collect().num_rows >= 0
