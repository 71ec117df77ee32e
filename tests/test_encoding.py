"""Encodings: vocab sizes and layouts of every mode, round trips, the 1-token map,
and the process-wide selector."""
import numpy as np
import pytest

from sigma0_b200.encoding import (get_tokenizer, set_token_mode, get_token_mode, Message_Tokenizer, Vocab,
                                  NA_VAL, START_TOK)
from sigma0_b200.encoding import tok1
from sigma0_b200.data import generate_day


@pytest.mark.parametrize("mode,vocab,msg_len", [("22tok", 12012, 22), ("23tok", 2114, 23),
                                                ("24tok", 2112, 24), ("26tok", 2112, 26)])
def test_vocab_and_len(mode, vocab, msg_len):
    t = get_tokenizer(mode)
    assert len(t.vocab) == vocab
    assert t.MSG_LEN == msg_len


@pytest.mark.parametrize("mode", ["22tok", "23tok", "24tok", "26tok"])
def test_roundtrip_synthetic(mode):
    t = get_tokenizer(mode)
    d = generate_day(300, seed=5)
    m = d.msgs.copy()
    m[:, 5] = np.minimum(m[:, 5], 9999)
    toks = t.encode_msgs(m)
    assert toks.shape == (300, t.MSG_LEN)
    assert toks.min() >= 0 and toks.max() < len(t.vocab)
    dec = t.decode_msgs(toks)
    cols = [1, 2, 4, 5, 6, 7, 8, 9]
    np.testing.assert_array_equal(dec[:, cols], m[:, cols])
    ref = m[:, 10] != NA_VAL
    np.testing.assert_array_equal(dec[ref][:, 10:14], m[ref][:, 10:14])


def test_22tok_known_ids():
    t = get_tokenizer("22tok")
    v = t.vocab
    assert v.field_range("time") == (4, 1004)
    assert v.field_range("event_type") == (1004, 1008)
    assert v.field_range("size") == (1008, 11008)
    assert v.field_range("price") == (11008, 12008)
    assert v.field_range("sign") == (12008, 12010)
    assert v.field_range("direction") == (12010, 12012)
    msg = np.array([[1, 1, 1, 0, -5, 120, 0, 123456789, 36000, 5000, NA_VAL, NA_VAL, NA_VAL, NA_VAL]])
    tk = t.encode_msgs(msg)[0]
    assert tk[0] == 1004 and tk[1] == 12011 and tk[2] == 12008 and tk[3] == 11013 and tk[4] == 1128


def test_1tok_map_roundtrip():
    t = get_tokenizer("24tok")
    toks = t.encode_msgs(generate_day(50, seed=1).msgs)
    loc = tok1.global_to_local(toks)
    assert (loc < np.array(tok1.FIELD_VOCAB_SIZES_WITH_SPECIAL)).all()
    np.testing.assert_array_equal(tok1.local_to_global(loc), toks)
    assert tok1.N_FIELDS == 24


def test_selector_proxies():
    set_token_mode("24tok")
    assert Message_Tokenizer.MSG_LEN == 24 and len(Vocab()) == 2112
    set_token_mode("22tok")
    assert Message_Tokenizer.MSG_LEN == 22 and get_token_mode() == "22tok"
    with pytest.raises(ValueError):
        set_token_mode("25tok")
    assert get_token_mode() == "22tok"
    set_token_mode("26tok")
