"""Seeded synthetic token sources.

* ``UniformBOSStream``: tokens uniform over the vocabulary with a BOS every ``bos_every`` tokens.
* ``ZipfDocumentSource``: documents of geometric length (mean ``mean_len``) whose tokens follow a
  Zipf(s) law over the non-special vocabulary; documents are BOS-prefixed by the packer.
* ``make_token_bytes``: seeded per-token UTF-8 byte lengths in ``[1, max_bytes]``; special tokens
  (BOS) get 0 bytes and are excluded from bits-per-byte, as in the reference's
  ``token_bytes.bin`` (scripts/prepare_wasm.ts:114-155) and ``evaluateBPB``
  (src/data/dataloader.ts:533-539).

The BOS id is ``vocab_size - 1``: it stays inside the embedding table, unlike the reference's
default ``bosTokenId = vocabSize`` (src/distributed/trainer.ts:94).
"""
from __future__ import annotations

import numpy as np


def bos_id(vocab_size: int) -> int:
    return vocab_size - 1


def make_token_bytes(vocab_size: int, max_bytes: int, seed: int = 1234) -> np.ndarray:
    rng = np.random.default_rng(seed)
    tb = rng.integers(1, max_bytes + 1, size=vocab_size, dtype=np.int32)
    tb[bos_id(vocab_size)] = 0
    return tb


class UniformBOSStream:
    """Infinite stream: uniform ids in [0, V-1) with BOS at every multiple of ``bos_every``."""

    def __init__(self, vocab_size: int, bos_every: int = 64, seed: int = 0):
        self.V = vocab_size
        self.bos_every = bos_every
        self.rng = np.random.default_rng(seed)
        self.pos = 0

    def take(self, n: int) -> np.ndarray:
        out = self.rng.integers(0, self.V - 1, size=n, dtype=np.int32)
        idx = np.arange(self.pos, self.pos + n)
        out[idx % self.bos_every == 0] = bos_id(self.V)
        self.pos += n
        return out


class ZipfDocumentSource:
    """Infinite seeded source of documents (without BOS) with Zipf(s)-distributed tokens."""

    def __init__(self, vocab_size: int, s: float = 1.1, mean_len: int = 512, seed: int = 0,
                 max_len: int | None = None, table_seed: int | None = None):
        self.V = vocab_size
        self.rng = np.random.default_rng(seed)
        n = vocab_size - 1  # BOS excluded
        ranks = np.arange(1, n + 1, dtype=np.float64)
        w = ranks ** (-s)
        self.cdf = np.cumsum(w / w.sum())
        self.cdf[-1] = 1.0
        # seeded rank -> id permutation so frequent ids are spread over the table
        ts = seed if table_seed is None else table_seed  # the permutation is the distribution, not the sample
        self.perm = np.random.default_rng(ts ^ 0x5EED).permutation(n).astype(np.int32)
        self.p_geom = 1.0 / mean_len
        self.max_len = max_len

    def sample_tokens(self, n: int) -> np.ndarray:
        u = self.rng.random(n)
        return self.perm[np.searchsorted(self.cdf, u, side="right").clip(max=len(self.perm) - 1)]

    def documents(self, count: int) -> list[np.ndarray]:
        lens = self.rng.geometric(self.p_geom, size=count)
        if self.max_len:
            lens = np.minimum(lens, self.max_len)
        toks = self.sample_tokens(int(lens.sum()))
        out = []
        o = 0
        for L in lens:
            out.append(toks[o:o + L])
            o += L
        return out

    def flat_with_offsets(self, count: int) -> tuple[np.ndarray, np.ndarray]:
        """``count`` documents as one int32 array plus int64 offsets (len count+1)."""
        lens = self.rng.geometric(self.p_geom, size=count)
        if self.max_len:
            lens = np.minimum(lens, self.max_len)
        toks = self.sample_tokens(int(lens.sum())).astype(np.int32)
        offs = np.zeros(count + 1, dtype=np.int64)
        np.cumsum(lens, out=offs[1:])
        return toks, offs
