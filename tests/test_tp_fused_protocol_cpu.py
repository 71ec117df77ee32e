"""Fake-rank simulation of the fused tensor-parallel GEMM + all-reduce protocol
(csrc/tp_fused.cu) on the CPU: the kernel's own index arithmetic, replayed for every
rank of a group, must deliver the sum over ranks of every output row to every rank,
write each receive slot row exactly once, and never address past the slots that
``FusedRowParallel`` allocates."""
import numpy as np
import pytest

BM = 128


def _rows_own(M, world):
    """FusedRowParallel's slot height: row tiles dealt round robin, rounded up."""
    tiles = -(-M // BM)
    return -(-tiles // world) * BM


def _simulate(M, N, world, seed=0):
    rng = np.random.default_rng(seed)
    parts = rng.standard_normal((world, M, N)).astype(np.float32)     # y_r @ w_r of every rank
    rows_own = _rows_own(M, world)
    tiles_m = M // BM
    recv = np.full((world, world * rows_own, N), np.nan, dtype=np.float32)
    writes = np.zeros((world, world * rows_own), dtype=np.int64)
    # phase 1: every rank stores each of its row tiles into the owner's slot for that rank
    for rank in range(world):
        for tm in range(tiles_m):
            owner, lt = tm % world, tm // world
            dst = rank * rows_own + lt * BM
            assert dst + BM <= world * rows_own
            recv[owner, dst:dst + BM] = parts[rank, tm * BM:(tm + 1) * BM]
            writes[owner, dst:dst + BM] += 1
    # phase 3: each owner sums its slots for its owned rows and stores them to every rank
    out = np.full((world, M, N), np.nan, dtype=np.float32)
    gathered = np.zeros((world, M), dtype=np.int64)
    for rank in range(world):
        owned_tiles = (tiles_m - rank + world - 1) // world
        for lrow in range(owned_tiles * BM):
            row = (rank + (lrow // BM) * world) * BM + lrow % BM
            acc = sum(recv[rank, k * rows_own + lrow] for k in range(world))
            for kk in range(world):
                out[kk, row] = acc
                gathered[kk, row] += 1
    return parts, out, writes, gathered, rows_own


@pytest.mark.parametrize("M,world", [(128, 1), (512, 2), (640, 2), (1280, 4), (1152, 8), (128 * 13, 8), (256, 8)])
def test_every_row_reduced_and_gathered_once(M, world):
    parts, out, writes, gathered, rows_own = _simulate(M, 16, world, seed=M + world)
    ref = parts.sum(0)
    for r in range(world):
        np.testing.assert_allclose(out[r], ref, rtol=1e-5, atol=1e-5)
    assert (gathered == 1).all()
    # every slot row is written at most once, and exactly once where an owned tile maps
    assert writes.max() <= 1
    tiles_m = M // BM
    for owner in range(world):
        owned = (tiles_m - owner + world - 1) // world
        for rank in range(world):
            block = writes[owner, rank * rows_own:rank * rows_own + owned * BM]
            assert (block == 1).all()


def test_slot_height_matches_the_module():
    """The Python helper sizes the slots with the same formula the simulation checks."""
    pytest.importorskip("torch")
    import sigma0_b200.parallel.tp_fused as tf
    for M in (100, 128, 300, 1000, 4096):
        for world in (1, 2, 4, 8):
            Mp = tf._ceil(M, tf.BM)
            rows_own = tf._ceil(Mp // tf.BM, world) // world * tf.BM
            assert rows_own == _rows_own(Mp, world)
            assert rows_own * world >= Mp
