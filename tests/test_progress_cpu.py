"""Progress messages: plain stderr lines off a terminal (tag and GPU prefix), a line per tenth."""

import pytest

from quail_b200.utils import progress


def test_plain_lines_with_tag_and_gpu(capsys, monkeypatch):
    monkeypatch.setenv(progress.LOG_TAG_ENV, "q7")
    monkeypatch.delenv("QUAIL_QUIET", raising=False)
    progress.set_gpu_index(3)
    try:
        progress.say("reading documents")
        progress.say("12 passes", detail=True)
        with progress.count("filter over 20 documents", 20, " docs") as c:
            for _ in range(20):
                c.advance()
    finally:
        progress.set_gpu_index(None)
    out = capsys.readouterr()
    assert out.out == ""                                  # stdout stays the caller's
    lines = out.err.strip().splitlines()
    assert all("[quail][q7][GPU 3]" in ln for ln in lines)
    assert any("reading documents" in ln for ln in lines) and any("12 passes" in ln for ln in lines)
    tenths = [ln for ln in lines if "docs (" in ln]
    assert len(tenths) == 10 and "20/20 docs" in tenths[-1]
    assert "20 docs in" in lines[-1]


def test_quiet(capsys, monkeypatch):
    monkeypatch.setenv("QUAIL_QUIET", "1")
    progress.say("nothing")
    assert capsys.readouterr().err == ""


@pytest.mark.parametrize("total", [0, 3])
def test_small_counts(capsys, total, monkeypatch):
    monkeypatch.delenv("QUAIL_QUIET", raising=False)
    with progress.count("x", total) as c:
        for _ in range(total):
            c.advance()
    assert f"x: {total} in" in capsys.readouterr().err
