"""LOBSTER import, day files, level selection and samplers."""
import os

import numpy as np
import pytest

from sigma0_b200.data.lobster import (lobster_day_from_arrays, raw_to_engine, resolve_day_files, save_day,
                                      select_levels, WindowSampler, ticker_balanced_order)


def _lobster_view(day, n):
    """Synthetic day -> LOBSTER columns (messages 0..n-1, book after each message)."""
    m = day.msgs[:n]
    t = [f"{s}.{ns:09d}" for s, ns in zip(m[:, 8], m[:, 9])]
    book_after = day.books[1:n + 1, 3:].astype(np.int64)
    return t, m[:, 1], m[:, 0], day.engine_msgs[:n, 2], m[:, 3], m[:, 2] * 2 - 1, book_after


def test_import_reproduces_engine_stream_and_books():
    from sigma0_b200.data.synthetic import generate_day
    from sigma0_b200.engine.book import book_from_l2
    day = generate_day(200, seed=7)
    n = 150
    lob = lobster_day_from_arrays(*_lobster_view(day, n))
    # the book before message i (i >= 1) is the synthetic day's book before message i
    assert np.array_equal(lob.books[1:, 3:], day.books[1:n, 3:])
    em = lob.engine_msgs
    assert np.array_equal(em[:, [0, 1, 3, 4, 6, 7]], day.engine_msgs[:n, [0, 1, 3, 4, 6, 7]])
    # cancel/execution references point at the original submission's time
    sub = {int(r[0]): (int(r[8]), int(r[9])) for r in lob.msgs if r[1] == 1}
    for r in lob.msgs:
        if r[1] in (2, 3, 4) and int(r[0]) in sub:
            assert (r[12], r[13]) == sub[int(r[0])]
    # replaying the imported stream from the opening book reproduces the recorded books
    ob = book_from_l2(day.l2_init)
    for i in range(n - 1):
        ob.process(em[i])
        assert np.array_equal(ob.l2(10), lob.books[i + 1, 3:].astype(np.int64))


def test_raw_to_engine_layout():
    raw = np.array([[17, 1, 1, 1_000_100, 1, 50, 0, 5, 34200, 7, -9999, -9999, -9999, -9999]])
    assert raw_to_engine(raw).tolist() == [[1, 1, 50, 1_000_100, 17, 0, 34200, 7]]


def test_resolve_and_select(tmp_path):
    from sigma0_b200.data.synthetic import generate_day
    d = generate_day(20, seed=1)
    from sigma0_b200.data.lobster import LobDay
    day = LobDay(d.msgs, d.books, d.engine_msgs, d.l2_init)
    save_day(day, str(tmp_path / "GOOG"), "GOOG", "2022-01-03")
    save_day(day, str(tmp_path / "GOOG"), "GOOG", "2022-01-05")
    save_day(day, str(tmp_path / "MSFT"), "MSFT", "2022-01-04")
    got = resolve_day_files(str(tmp_path), tickers=["GOOG", "MSFT"], date_range=("2022-01-03", "2022-01-04"))
    assert [os.path.basename(a) for a, _ in got] == ["GOOG_2022-01-03_message.npy", "MSFT_2022-01-04_message.npy"]
    wide = np.arange(2 * 40).reshape(2, 40)
    assert select_levels(wide, 3).shape == (2, 12)
    with pytest.raises(ValueError, match="divisible by 4"):
        select_levels(np.zeros((1, 38)), 2)


def test_window_sampler_interleave_and_resume():
    s0 = WindowSampler(20, batch=2, world=2, rank=0, seed=3)
    s1 = WindowSampler(20, batch=2, world=2, rank=1, seed=3)
    it0, it1 = iter(s0), iter(s1)
    e0 = sum((next(it0) for _ in range(5)), [])
    e1 = sum((next(it1) for _ in range(5)), [])
    assert sorted(e0 + e1) == list(range(20))          # one epoch covers every window once
    r = WindowSampler(20, batch=2, world=2, rank=0, seed=3, start_step=3)
    assert next(iter(r)) == e0[6:8]                    # resume continues with the next unseen batch
    order = ticker_balanced_order(["A", "A", "A", "B", "B", "C"], seed=0)
    assert sorted(order.tolist()) == list(range(6))
    first = [["A", "A", "A", "B", "B", "C"][i] for i in order[:3]]
    assert sorted(first) == ["A", "B", "C"]


def test_data_index_and_memory_mapped_days(tmp_path, monkeypatch):
    """With a data index the day files come from it (the tree is not walked), and the CLI's
    day loader memory-maps the arrays and builds engine rows only when asked."""
    import sigma0_b200.data.lobster as L
    from sigma0_b200.cli.common import load_days
    from sigma0_b200.data.synthetic import make_sequences
    d = make_sequences(1, 50, seed=3)[0]
    day = L.LobDay(d.msgs, d.books, d.engine_msgs, d.l2_init)
    for t, date in (("GOOG", "2022-01-03"), ("GOOG", "2022-01-05"), ("MSFT", "2022-01-04")):
        save_day(day, str(tmp_path / t), t, date)
    walked = resolve_day_files(str(tmp_path))
    idx = L.build_index(str(tmp_path))
    assert len(idx["shapes"]) == 6 and list(idx["shapes"].values())[0][0] == 50
    monkeypatch.setattr(L.os, "walk", lambda *a, **k: (_ for _ in ()).throw(AssertionError("walked")))
    assert resolve_day_files(str(tmp_path)) == walked
    assert len(resolve_day_files(str(tmp_path), tickers=["MSFT"])) == 1
    days = load_days(str(tmp_path), 0, 0, 0)
    assert len(days) == 3 and isinstance(days[0].msgs, np.memmap) and days[0]._engine is None
    assert np.array_equal(days[0].engine_msgs, raw_to_engine(np.asarray(d.msgs)))
    assert np.array_equal(days[0].l2_init, np.asarray(d.books[0, 3:], np.int64))
