"""NanoLLM's character vocabulary and text I/O (Examples/NanoLLM/NanoLLM.cpp:
95-206), for end-to-end text generation around the decode engine.

* The vocabulary is the corpus's distinct bytes sorted as C++ ``char`` --
  signed on the reference's x86 toolchains, so bytes 0x80-0xFF sort before
  0x00-0x7F (``BuildVocab``, :121-144); token id = position in that list.
* ``encode`` maps each byte to its id, unknown bytes to 0 (``std::map::
  operator[]`` default-inserts 0, :146-155).
* ``decode`` maps ids back to bytes, unknown ids to NUL (the same
  default-insert, :157-166); ``decode_tokens`` is ``DecodeMatrixTokens`` on a
  column of ids, unknown ids to ``?`` (:168-188).
"""
from __future__ import annotations

import numpy as np


def _signed_order(b: int) -> int:
    return b - 256 if b >= 128 else b


class CharVocab:
    def __init__(self, corpus: bytes):
        corpus = bytes(corpus)
        self.unique = bytes(sorted(set(corpus), key=_signed_order))
        self._to_id = np.zeros(256, np.uint32)
        for i, b in enumerate(self.unique):
            self._to_id[b] = i
        self.ids = self._to_id[np.frombuffer(corpus, np.uint8)] if corpus else np.zeros(0, np.uint32)

    @classmethod
    def from_file(cls, path: str) -> "CharVocab":
        """``LoadTextFile`` (:103-119) + ``BuildVocab``: the file's bytes."""
        with open(path, "rb") as f:
            return cls(f.read())

    @property
    def size(self) -> int:
        return len(self.unique)

    def encode(self, text) -> np.ndarray:
        data = text.encode("latin-1") if isinstance(text, str) else bytes(text)
        return self._to_id[np.frombuffer(data, np.uint8)] if data else np.zeros(0, np.uint32)

    def decode(self, ids) -> bytes:
        ids = np.asarray(ids, np.int64).ravel()
        table = np.frombuffer(self.unique, np.uint8)
        ok = (ids >= 0) & (ids < self.size)
        out = np.zeros(ids.size, np.uint8)
        out[ok] = table[ids[ok]]
        return out.tobytes()

    def decode_tokens(self, ids) -> bytes:
        ids = np.asarray(ids, np.int64).ravel()
        table = np.frombuffer(self.unique, np.uint8)
        ok = (ids >= 0) & (ids < self.size)
        out = np.full(ids.size, ord("?"), np.uint8)
        out[ok] = table[ids[ok]]
        return out.tobytes()
