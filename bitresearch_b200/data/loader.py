"""Token batching: flat-stream loader and BOS best-fit document packing.

* ``TokenDataLoader`` mirrors src/data/dataloader.ts:108-324: next-token batches from a flat int32
  stream with wrap-around (``next_batch``), a train/val split (``val_split``), fixed batches from an
  array (``batch_from_array``, ``get_fixed_batch``), and a document mode backed by the packer.
* ``BestFitDocumentBatcher`` mirrors src/data/bestFitPacking.ts:40-177: every row starts at a
  BOS-prefixed document; the row (capacity T+1) takes the largest buffered document that fits,
  otherwise the shortest one cropped to the remaining space; the buffer holds ``buffer_size``
  documents. The packing loop runs in C++ (``csrc/data/packer.cpp``) when the native module is
  built; the Python loop below is the oracle for it and the fallback on machines without the build.
* ``load_tokens_bin`` reads the reference's ``tokens.bin`` format (raw little-endian int32).
"""
from __future__ import annotations

from collections import deque
from typing import Callable, Sequence

import numpy as np


def load_tokens_bin(path: str) -> np.ndarray:
    return np.fromfile(path, dtype="<i4").astype(np.int32)


def load_token_bytes(path: str, vocab_size: int) -> np.ndarray:
    """``token_bytes`` as int32 [V]: ``.bin`` (int32) or ``.json`` (list); missing -> all ones
    (the reference's fallback, dataloader.ts:474-488)."""
    if not path:
        return np.ones(vocab_size, dtype=np.int32)
    if path.endswith(".json"):
        import json
        with open(path) as f:
            return np.asarray(json.load(f), dtype=np.int32)
    return np.fromfile(path, dtype="<i4").astype(np.int32)


# ------------------------------------------------------------------ manifest-aware discovery
# The reference looks for a parity manifest (explicit URL, else <artifact base>/manifest.json), takes
# every .bin shard it lists from <parity>/bin/, concatenates them into one token stream, and looks for
# token_bytes.bin / token-bytes.bin / token_bytes.json under <parity>/tokenizer/ then <parity>/bin/
# (trainer.ts:182-279, :489-511); without a manifest it tries tokens.bin at the data root and finally
# falls back to synthetic batches (trainer.ts:513-562). Here the locations are filesystem paths.
TOKEN_BYTES_NAMES = ("token_bytes.bin", "token-bytes.bin", "token_bytes.json")


def is_manifest(path: str) -> bool:
    """A parity manifest is a JSON object with a ``files`` entry; a token or document payload is not."""
    with open(path, "rb") as f:
        head = f.read(1 << 16).decode("utf-8", "ignore")
    return head.lstrip().startswith("{") and '"files"' in head


def find_manifest(path: str) -> str | None:
    """A manifest.json: ``path`` itself, or ``path/manifest.json``, or ``path/parity/manifest.json``."""
    import os
    if not path:
        return None
    if os.path.isfile(path) and path.endswith(".json"):
        return path if is_manifest(path) else None
    if os.path.isdir(path):
        for rel in ("manifest.json", os.path.join("parity", "manifest.json")):
            cand = os.path.join(path, rel)
            if os.path.isfile(cand):
                return cand
    return None


def manifest_artifacts(manifest_path: str) -> dict:
    """Resolves a parity manifest to local files: {"bin": [paths], "token_bytes": path | None,
    "tokenizer": path | None}. Shards are looked up under <manifest dir>/bin, then the manifest's
    recorded source directory."""
    import json
    import os
    with open(manifest_path) as f:
        m = json.load(f)
    root = os.path.dirname(os.path.abspath(manifest_path))
    src = m.get("source", {}) or {}
    bin_dirs = [os.path.join(root, "bin")] + ([src["binDir"]] if src.get("binDir") else [])
    tok_dirs = [os.path.join(root, "tokenizer")] + ([src["tokenizerDir"]] if src.get("tokenizerDir") else [])
    bins = []
    for name in (m.get("files", {}) or {}).get("bin", []):
        if not name.endswith(".bin"):
            continue
        for d in bin_dirs:
            cand = os.path.join(d, name)
            if os.path.isfile(cand):
                bins.append(cand)
                break
    token_bytes = tokenizer = None
    for d in tok_dirs + bin_dirs:
        for name in TOKEN_BYTES_NAMES:
            cand = os.path.join(d, name)
            if token_bytes is None and os.path.isfile(cand):
                token_bytes = cand
        cand = os.path.join(d, "tokenizer.json")
        if tokenizer is None and os.path.isfile(cand):
            tokenizer = cand
    return {"bin": bins, "token_bytes": token_bytes, "tokenizer": tokenizer}


def load_token_data(path: str) -> np.ndarray:
    """The token stream behind ``path``: a .bin shard, a manifest (all listed shards concatenated in
    order), or a directory holding a manifest or tokens.bin."""
    import os
    man = find_manifest(path)
    if man is not None:
        bins = manifest_artifacts(man)["bin"]
        if not bins:
            raise FileNotFoundError(f"manifest {man} lists no .bin shard that exists locally")
        return np.concatenate([load_tokens_bin(b) for b in bins])
    if os.path.isdir(path):
        cand = os.path.join(path, "tokens.bin")
        if os.path.isfile(cand):
            return load_tokens_bin(cand)
        raise FileNotFoundError(f"{path}: no manifest.json, parity/manifest.json or tokens.bin")
    return load_tokens_bin(path)


def load_json_payload(path: str) -> tuple[str, object]:
    """A JSON data file as ``("tokens", int32 array)`` or ``("documents", [int32 arrays])``: a flat list
    of ids is a token stream, a list of lists is documents, ``{"documents": [...]}`` or ``{"tokens": [...]}``
    name their shape (the reference's 'auto' format detection, src/data/dataloader.ts:40-61, 140-170)."""
    import json
    with open(path) as f:
        payload = json.load(f)
    if isinstance(payload, dict):
        if isinstance(payload.get("documents"), list):
            payload = payload["documents"]
        elif isinstance(payload.get("tokens"), list):
            return "tokens", np.asarray(payload["tokens"], dtype=np.int32)
        else:
            raise ValueError(f"{path}: unsupported JSON data shape; expected tokens or documents")
    if not isinstance(payload, list):
        raise ValueError(f"{path}: unsupported JSON data shape; expected tokens or documents")
    if payload and all(isinstance(d, list) for d in payload):
        return "documents", [np.asarray(d, dtype=np.int32) for d in payload]
    return "tokens", np.asarray(payload, dtype=np.int32)


def discover_token_bytes(path: str) -> str:
    """token_bytes next to the data of ``path`` (manifest locations, then the data directory); "" if none."""
    import os
    man = find_manifest(path)
    if man is not None:
        return manifest_artifacts(man)["token_bytes"] or ""
    d = path if os.path.isdir(path) else os.path.dirname(path)
    for name in TOKEN_BYTES_NAMES:
        cand = os.path.join(d, name)
        if d and os.path.isfile(cand):
            return cand
    return ""


class TokenDataLoader:
    def __init__(self, tokens: np.ndarray | None = None):
        self.tokens = np.zeros(0, np.int32) if tokens is None else np.ascontiguousarray(tokens, np.int32)
        self.pos = 0
        self.epochs = 0

    def set_token_stream(self, tokens: Sequence[int]) -> None:
        self.tokens = np.ascontiguousarray(tokens, np.int32)
        self.pos = 0
        self.epochs = 0

    @property
    def num_tokens(self) -> int:
        return len(self.tokens)

    def next_batch(self, batch: int, seq: int) -> tuple[np.ndarray, np.ndarray]:
        """dataloader.ts:225-249: targets wrap to tokens[0] at the end of the stream."""
        n = batch * seq
        if len(self.tokens) == 0:
            raise RuntimeError("TokenDataLoader has no token stream loaded.")
        L = len(self.tokens)
        idx = (self.pos + np.arange(n)) % L
        self.epochs += (self.pos + n) // L
        self.pos = (self.pos + n) % L
        nxt = idx + 1
        targets = np.where(nxt >= L, self.tokens[0], self.tokens[np.minimum(nxt, L - 1)])
        return self.tokens[idx].reshape(batch, seq), targets.astype(np.int32).reshape(batch, seq)

    def val_split(self, ratio: float = 0.1) -> np.ndarray:
        split = int(len(self.tokens) * (1 - ratio))
        val = self.tokens[split:].copy()
        self.tokens = self.tokens[:split]
        self.pos = 0
        return val

    @staticmethod
    def batch_from_array(tokens: np.ndarray, batch: int, seq: int, offset: int) -> tuple[np.ndarray, np.ndarray]:
        n = batch * seq
        if len(tokens) == 0:
            return np.zeros((batch, seq), np.int32), np.zeros((batch, seq), np.int32)
        L = len(tokens)
        base = offset % L
        idx = (base + np.arange(n)) % L
        return tokens[idx].reshape(batch, seq), tokens[(idx + 1) % L].reshape(batch, seq)

    def get_fixed_batch(self, batch: int, seq: int, start: int) -> tuple[np.ndarray, np.ndarray]:
        return self.batch_from_array(self.tokens, batch, seq, start)


def split_documents(docs: list, ratio: float = 0.1) -> tuple[list, list]:
    split = int(len(docs) * (1 - ratio))
    return docs[:split], docs[split:]


class BestFitDocumentBatcher:
    """Python restatement of the reference packer; ``next_batch`` returns (inputs, targets, epoch).

    ``source`` is either a finite list of documents (cycled with epoch counting, as in the
    reference) or a callable ``source(n) -> list[np.ndarray]`` producing fresh documents.
    """

    def __init__(self, source: list | Callable[[int], list], bos_id: int, buffer_size: int = 1000,
                 documents_are_bos_prefixed: bool = False):
        self.bos = bos_id
        self.buffer_size = max(1, buffer_size)
        self.prefixed = documents_are_bos_prefixed
        self.source = source
        self.src_idx = 0
        self.epoch = 1
        self.buffer: list[np.ndarray] = []
        self._pending: deque = deque()

    def _prep(self, d) -> np.ndarray:
        d = np.asarray(d, dtype=np.int32)
        if self.prefixed:
            return d
        return np.concatenate([np.array([self.bos], np.int32), d])

    def _take(self) -> np.ndarray:
        if callable(self.source):
            if not self._pending:
                self._pending.extend(self.source(max(self.buffer_size, 256)))
            return self._prep(self._pending.popleft())
        if len(self.source) == 0:
            raise RuntimeError("BestFitDocumentBatcher requires at least one document.")
        if self.src_idx >= len(self.source):
            self.src_idx = 0
            self.epoch += 1
        d = self.source[self.src_idx]
        self.src_idx += 1
        return self._prep(d)

    def pack_rows(self, batch: int, seq: int) -> np.ndarray:
        cap = seq + 1
        rows = np.empty((batch, cap), np.int32)
        for r in range(batch):
            pos = 0
            while pos < cap:
                while len(self.buffer) < self.buffer_size:
                    self.buffer.append(self._take())
                rem = cap - pos
                best, best_len = -1, 0
                for i, d in enumerate(self.buffer):
                    if best_len < len(d) <= rem:
                        best, best_len = i, len(d)
                if best >= 0:
                    d = self.buffer.pop(best)
                    rows[r, pos:pos + len(d)] = d
                    pos += len(d)
                    continue
                si = min(range(len(self.buffer)), key=lambda i: (len(self.buffer[i]), i))
                d = self.buffer.pop(si)
                rows[r, pos:cap] = d[:rem]
                pos = cap
        return rows

    def next_batch(self, batch: int, seq: int):
        rows = self.pack_rows(batch, seq)
        return rows[:, :seq].copy(), rows[:, 1:].copy(), self.epoch
