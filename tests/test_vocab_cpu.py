"""NanoLLM's character vocabulary and text I/O (freeml_b200/vocab.py) against
the reference's own BuildVocab / encode / decode / DecodeMatrixTokens
(Examples/NanoLLM/NanoLLM.cpp:95-206), whose outputs on a synthetic corpus are
committed in tests/golden/vocab.npz (tests/golden/make_golden.py vocab)."""
import os

import numpy as np
import pytest

from freeml_b200.vocab import CharVocab

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def g():
    return np.load(os.path.join(HERE, "golden", "vocab.npz"))


def test_vocabulary_order_and_corpus_ids(g):
    """Distinct bytes in signed-char order (0xC0.. before ASCII), ids = rank."""
    v = CharVocab(g["corpus"].tobytes())
    assert v.unique == g["unique"].tobytes()
    assert v.size == g["unique"].size
    assert v.unique[0] >= 0x80 and v.unique[-1] < 0x80
    np.testing.assert_array_equal(v.ids, g["corpus_ids"])


def test_encode_maps_unknown_bytes_to_zero(g):
    v = CharVocab(g["corpus"].tobytes())
    enc = v.encode(g["text"].tobytes())
    np.testing.assert_array_equal(enc, g["encode"])
    absent = set(g["text"].tolist()) - set(g["corpus"].tolist())
    assert absent, "the fixture text must hold bytes the corpus lacks"


def test_decode_and_decode_tokens(g):
    v = CharVocab(g["corpus"].tobytes())
    assert v.decode(g["ids"]) == g["decode"].tobytes()          # unknown ids -> NUL
    assert v.decode_tokens(g["ids"]) == g["decode_tokens"].tobytes()  # unknown ids -> '?'
    assert (g["ids"] >= v.size).any()


def test_round_trip_and_edges(tmp_path):
    text = b"to be or not to be\n"
    p = tmp_path / "corpus.txt"
    p.write_bytes(text)
    v = CharVocab.from_file(str(p))
    assert v.decode(v.encode(text)) == text
    assert v.encode("not").tolist() == v.encode(b"not").tolist()
    empty = CharVocab(b"")
    assert empty.size == 0 and empty.ids.size == 0 and empty.encode(b"").size == 0
    assert empty.decode_tokens([0, 3]) == b"??"
