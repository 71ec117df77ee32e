"""bench.py's host-side configuration: the context-parallel sequence length per world size."""
from types import SimpleNamespace


def test_cp_messages_keep_the_per_rank_segment():
    import bench
    from sigma0_b200.models import preset_args
    h = preset_args("hybrid1b")
    assert [bench.cp_messages(h, n) for n in (1, 2, 4, 8)] == [375, 750, 1500, 3000]
    # NSA: a segment of whole messages that is also a whole number of 64-token selection blocks
    n = preset_args("nsa1b")
    for w in (1, 2, 4, 8):
        m = bench.cp_messages(n, w)
        assert m % w == 0 and (m // w * 22) % 64 == 0 and m >= 375 * w
    assert bench.cp_messages(SimpleNamespace(n_messages=16, architecture="mamba3", msg_len=22), 2) == 4
