"""Masking objectives, book ablations and the .npy / .npy.zst loader."""
import numpy as np
import pytest

from sigma0_b200.data import masks as M
from sigma0_b200.data.dataset import LobWindowDataset
from sigma0_b200.data.synthetic import generate_day
from sigma0_b200.encoding import HIDDEN_TOK, MASK_TOK, START_TOK, get_tokenizer


@pytest.fixture
def win():
    tok = get_tokenizer("22tok")
    d = generate_day(40, seed=1)
    return tok, tok.encode_msgs(d.msgs[:6])


def test_no_mask_variants(win):
    tok, seq = win
    (x, _), y = M.no_mask(seq)
    assert x[0] == START_TOK and (x[1:] == seq.reshape(-1)[:-1]).all() and (y == seq.reshape(-1)).all()
    (x1, _), y1 = M.no_mask_1tok(seq)
    assert (x1[0] == START_TOK).all() and (x1[1:] == seq[:-1]).all()
    (xi, _), _ = M.inference_mask(seq)
    assert xi.shape[0] == seq.size + 1


def test_masking_fn_fields_and_positions(win):
    tok, seq = win
    rng = np.random.default_rng(0)
    fn = M.masking_fn(tok, random_fields=["price"], randomize_message=False)
    a, b = M.field_slice(tok, tok.FIELDS.index("price"))
    for _ in range(20):
        s, y = fn(seq, rng)
        diff = np.argwhere(s != seq)
        assert len(diff) == 1 and diff[0][0] == seq.shape[0] - 1 and a <= diff[0][1] < b
        assert s[tuple(diff[0])] == MASK_TOK and y == seq[tuple(diff[0])]
    with pytest.raises(ValueError):
        M.masking_fn(tok)


def test_random_and_causal_masks(win):
    tok, seq = win
    rng = np.random.default_rng(3)
    for _ in range(50):
        s, y = M.random_mask(tok, seq, rng)
        last = s[-1]
        assert (last == MASK_TOK).sum() == 1 and (s[:-1] == seq[:-1]).all()
        t0, t1 = tok.TIME_START_I, tok.TIME_END_I + 1
        assert MASK_TOK not in last[t0:t1]
        assert y == seq[-1][np.argmax(last == MASK_TOK)]
    for sel in ("sequential_no_time", "sequential", "random", "unconditional"):
        for _ in range(30):
            s, y = M.causal_mask(tok, seq, rng, sel)
            i = int(np.argmax(s[-1] == MASK_TOK))
            assert (s[-1] == MASK_TOK).sum() == 1 and y == seq[-1][i]
            f = next(k for k in range(len(tok.FIELDS)) if M.field_slice(tok, k)[0] <= i < M.field_slice(tok, k)[1])
            a, b = M.field_slice(tok, f)
            assert (s[-1][i + 1:b] == HIDDEN_TOK).all()
            if sel == "sequential_no_time":
                assert tok.FIELDS[f] not in ("time_s", "time_ns")
                assert (s[-1][b:] == HIDDEN_TOK).all()


def test_book_ablations_and_dataset_objectives(tmp_path):
    b = np.random.default_rng(0).normal(size=(5, 9))
    assert (M.ablate_books(b, "zero", (0, 0)) == 0).all()
    n = M.ablate_books(b, "noise", (1, 2))
    assert (n[:, :3] == 0).all() and np.allclose(n, M.ablate_books(b, "noise", (1, 2)))
    sh = M.ablate_books(b, "shuffle", (1, 2))
    assert sorted(map(tuple, sh)) == sorted(map(tuple, b))
    with pytest.raises(ValueError):
        M.ablate_books(b, "bogus", (0, 0))
    days = [generate_day(60, seed=2)]
    ds = LobWindowDataset.from_days(days, 10, mask="causal", book_ablation="zero")
    x, y, bk = ds[0]
    assert x.shape[0] == 10 * 22 and y.dim() == 0 and (bk == 0).all()
    x2, y2, _ = ds[0]
    assert (x == x2).all() and y == y2                       # seeded per window
    xi, _, _ = LobWindowDataset.from_days(days, 10, mask="inference")[0]
    assert xi[0] == START_TOK and xi.shape[0] == 221
    # .npy wins over .npy.zst; a lone .npy.zst needs zstandard
    np.save(tmp_path / "a.npy", b)
    assert np.allclose(M.load_npy(str(tmp_path / "a.npy.zst")), b)
    (tmp_path / "c.npy.zst").write_bytes(b"\x28\xb5\x2f\xfd")
    with pytest.raises((ImportError, Exception)):
        M.load_npy(str(tmp_path / "c.npy.zst"))
