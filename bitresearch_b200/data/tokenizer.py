"""Byte-level BPE tokenizer of the data-preparation step (native trainer and encoder).

The reference trains rustbpe (a byte-level BPE) on text shards with the GPT-4 split pattern, a base
vocabulary of ``8192 - 4`` tokens and four reserved special tokens appended after it, the first of
which is BOS (scripts/prepare_wasm.ts:14-17, :114-155, :276-308). This module keeps those
conventions and artifact formats:

* pre-tokenization by the GPT-4 split regex (``regex`` module: Unicode classes and possessive
  quantifiers), then byte-level BPE inside each chunk;
* token id = merge rank: ids 0..255 are the bytes, id 256 + i is the i-th merge;
* specials ``<|reserved_0..3|>`` get ids ``vocab_size() .. vocab_size() + 3``; BOS is the first;
* ``tokenizer.json``: artifactVersion, name, pattern, vocabSize, fullVocabSize, numMerges,
  specialTokens, specialTokenIds, bosToken, bosTokenId, tokenBytesFile, mergeableRanksEncoding
  ("base64") and mergeableRanks ([base64 bytes, rank] pairs), as written at prepare_wasm.ts:130-146;
* ``token_bytes.bin``: int32 byte length of every token of the full vocabulary, 0 for specials
  (prepare_wasm.ts:121-150), the table ``evaluate_bpb`` divides by.

Training and encoding run in C++ (``_native_data.bpe_train`` / ``BPEEncoder``); equal pair counts
are broken towards the smaller (left, right) pair, so a training run is deterministic.
"""
from __future__ import annotations

import base64
import collections
import json
import os
import threading
from typing import Iterable, Sequence

import numpy as np

SPLIT_PATTERN = (r"""'(?i:[sdmt]|ll|ve|re)|[^\r\n\p{L}\p{N}]?+\p{L}+|\p{N}{1,2}| ?[^\s\p{L}\p{N}]++[\r\n]*|"""
                 r"""\s*[\r\n]|\s+(?!\S)|\s+""")
SPECIAL_TOKENS = ["<|reserved_0|>", "<|reserved_1|>", "<|reserved_2|>", "<|reserved_3|>"]
DEFAULT_VOCAB_SIZE = 8192  # full vocabulary, specials included


def _native():
    from .. import _native_data
    return _native_data


_SPLIT_TABLE = False
_SPLIT_LOCK = threading.Lock()


def _install_split_table() -> None:
    r"""Gives the native pre-split the class of every code point, taken from the regex engine itself
    (``\p{L}``, ``\p{N}``, ``\s``, and which code points match the contraction letters case-insensitively),
    so the native and regex splits agree by construction. Once per process, about 0.3 s."""
    global _SPLIT_TABLE
    with _SPLIT_LOCK:
        if not _SPLIT_TABLE:
            _build_split_table()
            _SPLIT_TABLE = True


def _build_split_table() -> None:
    import regex
    let, dig, nl, ws, oth, bad = range(6)
    allc = "".join(map(chr, range(0xD800))) + "".join(map(chr, range(0xE000, 0x110000)))
    t = np.full(0x110000, oth, dtype=np.uint8)
    t[0xD800:0xE000] = bad
    for cls, pat in ((ws, r"\s"), (let, r"\p{L}"), (dig, r"\p{N}")):
        t[np.fromiter(map(ord, regex.findall(pat, allc)), dtype=np.int64)] = cls
    t[[ord("\n"), ord("\r")]] = nl
    for k, ch in enumerate("sdmtlver"):
        t[np.fromiter(map(ord, regex.findall(f"(?i:{ch})", allc)), dtype=np.int64)] |= (k + 1) << 3
    _native().set_split_table(t)


class BPETokenizer:
    def __init__(self, merges: Sequence[tuple[int, int]] = (), pattern: str = SPLIT_PATTERN):
        import regex
        self.pattern = pattern
        self._re = regex.compile(pattern)
        self.merges = [tuple(map(int, m)) for m in merges]
        self.native_split = pattern == SPLIT_PATTERN
        if self.native_split:
            _install_split_table()
        self._enc = _native().BPEEncoder(self.merges) if self.merges else None
        self._tls = threading.local()  # one encoder per pool thread (an encoder's chunk cache is not shared)
        self._vocab_bytes: list[bytes] | None = None

    # ------------------------------------------------------------------ training
    def chunk_counts(self, texts: Iterable[str], pool=None, chunk: int = 2048) -> collections.Counter:
        """Occurrences of every pre-tokenized chunk; with a ``pool`` from :meth:`pool` the parts are split
        and counted on its threads (natively, without the GIL) and merged in order."""
        counts: collections.Counter = collections.Counter()
        if pool is None:
            texts = list(texts)
            native = _native().count_chunks_native(texts) if self.native_split else None
            if native is None:
                rest = range(len(texts))
            else:  # split and counted natively; texts the table cannot split go through the regex
                keys, cnts, rest = native
                for k, c in zip(keys, cnts):
                    counts[k.decode("utf-8")] += c
            for i in rest:
                counts.update(self._re.findall(texts[i]))
            return counts
        texts = list(texts)
        for part in pool.map(self.chunk_counts, [texts[i:i + chunk] for i in range(0, len(texts), chunk)]):
            counts.update(part)
        return counts

    def train(self, texts: Iterable[str], vocab_size_no_special: int, pool=None) -> "BPETokenizer":
        """Learns ``vocab_size_no_special - 256`` merges over the texts' chunks."""
        counts = self.chunk_counts(texts, pool=pool)
        chunks = [c.encode("utf-8") for c in counts]
        merges = _native().bpe_train(chunks, list(counts.values()), int(vocab_size_no_special))
        self.merges = [tuple(m) for m in merges]
        self._enc = _native().BPEEncoder(self.merges)
        self._tls = threading.local()
        self._vocab_bytes = None
        return self

    # ------------------------------------------------------------------ vocabulary
    def vocab_size(self) -> int:
        """Base vocabulary (bytes + merges), without the special tokens."""
        return 256 + len(self.merges)

    def num_merges(self) -> int:
        return len(self.merges)

    def full_vocab_size(self) -> int:
        return self.vocab_size() + len(SPECIAL_TOKENS)

    @property
    def bos_id(self) -> int:
        return self.vocab_size()

    def special_token_ids(self) -> dict[str, int]:
        return {t: self.vocab_size() + i for i, t in enumerate(SPECIAL_TOKENS)}

    def vocab_bytes(self) -> list[bytes]:
        if self._vocab_bytes is None:
            vb = [bytes([i]) for i in range(256)]
            for a, b in self.merges:
                vb.append(vb[a] + vb[b])
            self._vocab_bytes = vb
        return self._vocab_bytes

    def mergeable_ranks(self) -> list[tuple[bytes, int]]:
        return [(b, i) for i, b in enumerate(self.vocab_bytes())]

    def token_bytes(self) -> np.ndarray:
        """int32 byte length of every token of the full vocabulary (0 for the special tokens)."""
        tb = np.zeros(self.full_vocab_size(), dtype=np.int32)
        tb[:self.vocab_size()] = [len(b) for b in self.vocab_bytes()]
        return tb

    # ------------------------------------------------------------------ encode / decode
    def encode(self, text: str, _enc=None) -> np.ndarray:
        enc = _enc or self._enc
        if enc is None:
            raise RuntimeError("tokenizer has no merges: train or load it first")
        if self.native_split:
            ids = enc.encode_text(text)  # split natively unless the text holds a lone surrogate
            if ids is not None:
                return ids
        return enc.encode_chunks(self._re.findall(text))  # str chunks reach C++ as UTF-8 bytes

    def _encode_part(self, texts: list[str]) -> list[np.ndarray]:
        enc = getattr(self._tls, "enc", None)
        if enc is None:
            enc = self._tls.enc = _native().BPEEncoder(self.merges)
        return [self.encode(t, enc) for t in texts]

    def batch_encode(self, texts: Sequence[str], pool=None, chunk: int = 256) -> list[np.ndarray]:
        """Encodes ``texts`` in order; with a ``pool`` from :meth:`pool` the parts run on its threads, each
        with its own encoder (the native split and merge loop release the GIL)."""
        if pool is None or len(texts) <= chunk:
            return [self.encode(t) for t in texts]
        parts = [list(texts[i:i + chunk]) for i in range(0, len(texts), chunk)]
        return [ids for part in pool.map(self._encode_part, parts) for ids in part]

    def pool(self, workers: int):
        """A thread pool for :meth:`batch_encode` and :meth:`chunk_counts` (use it as a context manager)."""
        from concurrent.futures import ThreadPoolExecutor
        return ThreadPoolExecutor(max_workers=max(1, workers), thread_name_prefix="bpe")

    def decode(self, ids: Iterable[int]) -> str:
        vb = self.vocab_bytes()
        n = len(vb)
        return b"".join(vb[i] for i in ids if 0 <= i < n).decode("utf-8", errors="replace")

    # ------------------------------------------------------------------ artifacts
    def metadata(self) -> dict:
        return {
            "artifactVersion": 1,
            "name": "bitresearch-b200-bpe",
            "pattern": self.pattern,
            "vocabSize": self.vocab_size(),
            "fullVocabSize": self.full_vocab_size(),
            "numMerges": self.num_merges(),
            "specialTokens": list(SPECIAL_TOKENS),
            "specialTokenIds": self.special_token_ids(),
            "bosToken": SPECIAL_TOKENS[0],
            "bosTokenId": self.bos_id,
            "tokenBytesFile": "token_bytes.bin",
            "mergeableRanksEncoding": "base64",
            "mergeableRanks": [[base64.b64encode(b).decode("ascii"), r] for b, r in self.mergeable_ranks()],
        }

    def save(self, directory: str) -> tuple[str, str]:
        """Writes tokenizer.json and token_bytes.bin (atomically, through a temporary file)."""
        os.makedirs(directory, exist_ok=True)
        tj = os.path.join(directory, "tokenizer.json")
        tb = os.path.join(directory, "token_bytes.bin")
        _atomic_write(tj, (json.dumps(self.metadata(), indent=2) + "\n").encode())
        _atomic_write(tb, self.token_bytes().tobytes())
        return tj, tb

    @classmethod
    def load(cls, path: str) -> "BPETokenizer":
        """Loads tokenizer.json: the merges are rebuilt from the mergeable ranks."""
        with open(path) as f:
            meta = json.load(f)
        if meta.get("mergeableRanksEncoding", "base64") != "base64":
            raise ValueError("tokenizer.json: only base64 mergeable ranks are supported")
        ranks = sorted(((base64.b64decode(b), int(r)) for b, r in meta["mergeableRanks"]), key=lambda x: x[1])
        for i, (b, r) in enumerate(ranks[:256]):
            if r != i or b != bytes([i]):
                raise ValueError("tokenizer.json: ranks 0..255 must be the single bytes")
        # Token r came from merging the two tokens that the first r - 256 merges leave when they encode
        # r's own bytes; rebuilding in rank order reproduces the trained encoder exactly.
        merges: list[tuple[int, int]] = []
        pair_rank: dict[tuple[int, int], int] = {}
        for b, r in ranks[256:]:
            if r != 256 + len(merges):
                raise ValueError(f"tokenizer.json: ranks are not contiguous at {r}")
            ids = list(b)
            while len(ids) > 2:
                best = min(((pair_rank.get((ids[i], ids[i + 1]), 1 << 30), i) for i in range(len(ids) - 1)))
                if best[0] == 1 << 30:
                    break
                a, c = ids[best[1]], ids[best[1] + 1]
                nid, out, i = 256 + best[0], [], 0
                while i < len(ids):
                    if i + 1 < len(ids) and ids[i] == a and ids[i + 1] == c:
                        out.append(nid)
                        i += 2
                    else:
                        out.append(ids[i])
                        i += 1
                ids = out
            if len(ids) != 2:
                raise ValueError(f"tokenizer.json: token {r} is not a merge of two earlier tokens")
            pair_rank[(ids[0], ids[1])] = len(merges)
            merges.append((ids[0], ids[1]))
        return cls(merges, pattern=meta.get("pattern", SPLIT_PATTERN))


def _atomic_write(path: str, data: bytes) -> None:
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(data)
    os.replace(tmp, path)
