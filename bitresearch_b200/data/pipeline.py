"""Training/validation batch sources built from a :class:`TrainConfig`.

``make_batch_source(cfg, split, rank, world)`` returns an object with ``next(batch, seq)`` giving
host int32 ``(inputs, targets)`` arrays and an ``epoch`` attribute. Each rank draws from its own
seeded stream (seed, split and rank mixed), so data-parallel ranks see disjoint data, like separate
browser tabs in the reference. The validation split uses a different seed, i.e. a held-out stream.
The synthetic distribution itself (which id is frequent, the Markov successors) comes from a
separate table seed shared by all ranks and both splits.

``PinnedPrefetcher`` produces the next batch on a host thread into page-locked buffers and copies
it to the device on a side stream, so the host->device transfer overlaps the previous step.
"""
from __future__ import annotations

import math
import threading
from queue import Queue

import numpy as np
import torch

from ..config import TrainConfig
from .loader import BestFitDocumentBatcher, TokenDataLoader, find_manifest, load_json_payload, load_token_data
from .synthetic import UniformBOSStream, ZipfDocumentSource, bos_id


def _native():
    try:
        from .. import _native_data  # type: ignore
        return _native_data
    except Exception:
        return None


def _seed(cfg: TrainConfig, split: str, rank: int) -> int:
    """Sampling seed of one rank's stream of one split."""
    return (cfg.seed * 1_000_003 + (0 if split == "train" else 7_777_777) + rank * 9176) & 0x7FFFFFFF


def _table_seed(cfg: TrainConfig) -> int:
    """Seed of the token distribution itself (id permutation, Markov successors): one per run, shared
    by every rank and by the validation split."""
    return (cfg.seed * 2_654_435_761 + 0x51A7) & 0x7FFFFFFF


class _ZipfNative:
    def __init__(self, cfg: TrainConfig, seed: int):
        mod = _native()
        self.mod = mod
        if cfg.data == "markov":
            self.p = mod.markov_packer(cfg.model.vocab_size, cfg.zipf_s, float(cfg.doc_mean_len), seed,
                                       _table_seed(cfg), cfg.markov_p1, cfg.markov_p2, cfg.markov_branch,
                                       cfg.document_buffer_size, 0)
        else:
            self.p = mod.zipf_packer(cfg.model.vocab_size, cfg.zipf_s, float(cfg.doc_mean_len), seed,
                                     cfg.document_buffer_size, 0, _table_seed(cfg))

    @property
    def epoch(self):
        return self.p.epoch

    def next(self, batch: int, seq: int):
        rows = np.empty((batch, seq + 1), np.int32)
        self.mod.pack_rows(self.p, rows, batch, seq)
        return rows[:, :seq], rows[:, 1:]

    def next_into(self, inputs: torch.Tensor, targets: torch.Tensor, batch: int, seq: int):
        self.mod.pack_split(self.p, inputs.data_ptr(), targets.data_ptr(), batch, seq)


class _ZipfPython:
    def __init__(self, cfg: TrainConfig, seed: int):
        src = ZipfDocumentSource(cfg.model.vocab_size, cfg.zipf_s, cfg.doc_mean_len, seed,
                                 table_seed=_table_seed(cfg))
        self.b = BestFitDocumentBatcher(src.documents, bos_id(cfg.model.vocab_size), cfg.document_buffer_size)

    @property
    def epoch(self):
        return self.b.epoch

    def next(self, batch: int, seq: int):
        x, y, _ = self.b.next_batch(batch, seq)
        return x, y


class _Uniform:
    def __init__(self, cfg: TrainConfig, seed: int):
        self.s = UniformBOSStream(cfg.model.vocab_size, cfg.bos_every, seed)
        self.epoch = 0

    def next(self, batch: int, seq: int):
        rows = self.s.take(batch * (seq + 1)).reshape(batch, seq + 1)
        return rows[:, :seq].copy(), rows[:, 1:].copy()


class _Documents:
    """A finite document list, best-fit BOS packed (natively when the data module is built), cycled with
    an epoch counter like the reference's document loader (src/data/dataloader.ts:194-206)."""

    def __init__(self, docs: list, bos: int, buffer_size: int, prefixed: bool):
        if not docs:
            raise ValueError("no documents in this split")
        mod = _native()
        self.mod = mod
        if mod is not None:
            flat = np.concatenate(docs).astype(np.int32) if docs else np.zeros(0, np.int32)
            offs = np.zeros(len(docs) + 1, dtype=np.int64)
            np.cumsum([len(d) for d in docs], out=offs[1:])
            self.p = mod.corpus_packer(bos, buffer_size, flat, offs, prefixed)
            self.b = None
        else:
            self.b = BestFitDocumentBatcher(docs, bos, buffer_size, documents_are_bos_prefixed=prefixed)

    @property
    def epoch(self):
        return self.p.epoch if self.b is None else self.b.epoch

    def next(self, batch: int, seq: int):
        if self.b is not None:
            x, y, _ = self.b.next_batch(batch, seq)
            return x, y
        rows = np.empty((batch, seq + 1), np.int32)
        self.mod.pack_rows(self.p, rows, batch, seq)
        return rows[:, :seq], rows[:, 1:]


class _Tokens:
    def __init__(self, tokens: np.ndarray):
        self.l = TokenDataLoader(tokens)

    @property
    def epoch(self):
        return self.l.epochs

    def next(self, batch: int, seq: int):
        return self.l.next_batch(batch, seq)


def make_batch_source(cfg: TrainConfig, split: str = "train", rank: int = 0, world: int = 1, native: bool = True):
    seed = _seed(cfg, split, rank)
    if cfg.data == "zipf":
        if native and _native() is not None:
            return _ZipfNative(cfg, seed)
        return _ZipfPython(cfg, seed)
    if cfg.data == "markov":
        if _native() is None:
            raise RuntimeError("data=markov needs the native data module (python setup.py build_ext --inplace)")
        return _ZipfNative(cfg, seed)
    if cfg.data == "uniform":
        return _Uniform(cfg, seed)
    if cfg.data in ("tokens", "documents"):
        json_payload = cfg.data_path.endswith(".json") and find_manifest(cfg.data_path) is None
        kind, payload = (load_json_payload(cfg.data_path) if json_payload
                         else ("tokens", load_token_data(cfg.data_path)))
        if cfg.data == "documents" and kind != "documents":
            raise ValueError(f"{cfg.data_path}: data=documents needs a list of token arrays")
        if kind == "documents":  # split by document count (src/data/dataloader.ts:269-278)
            docs = payload
            split_at = int(len(docs) * (1 - cfg.val_fraction))
            part = docs[:split_at] if split == "train" else docs[split_at:]
            if split == "train" and world > 1:
                n = len(part) // world
                part = part[rank * n:(rank + 1) * n]
            bos = cfg.bos_token_id if cfg.bos_token_id >= 0 else cfg.model.vocab_size - 1
            return _Documents(part, bos, cfg.document_buffer_size, cfg.documents_bos_prefixed)
        toks = payload
        split_at = int(len(toks) * (1 - cfg.val_fraction))
        part = toks[:split_at] if split == "train" else toks[split_at:]
        if split == "train" and world > 1:  # contiguous per-rank shards of the training stream
            n = len(part) // world
            part = part[rank * n:(rank + 1) * n]
        return _Tokens(part)
    raise ValueError(f"unknown data source {cfg.data!r}")


def markov_floor(cfg: TrainConfig, token_bytes: np.ndarray, n_tokens: int, batch: int) -> tuple[float, float]:
    """Loss floor of ``data=markov`` on the validation stream: the exact negative log-likelihood of its
    first ``n_tokens`` targets under the generating process, as (bits per byte, nats per token). A model
    that had learned the process exactly would score this ``val_bpb``."""
    if cfg.data != "markov":
        raise ValueError("markov_floor needs data=markov")
    mod = _native()
    T = cfg.model.sequence_len
    src = _ZipfNative(cfg, _seed(cfg, "val", 0))
    rows = np.empty((batch, T + 1), np.int32)
    nats = nbytes = count = 0.0
    for _ in range(max(1, n_tokens // (batch * T))):
        mod.pack_rows(src.p, rows, batch, T)
        nll = mod.markov_nll(src.p, rows, batch, T)
        tb = token_bytes[rows[:, 1:]]
        keep = tb > 0
        nats += float(nll[keep].sum())
        nbytes += float(tb[keep].sum())
        count += float(keep.sum())
    return nats / (math.log(2) * nbytes), nats / count


class PinnedPrefetcher:
    """Host thread packs batches into pinned buffers; ``get()`` returns device tensors.

    The H2D copy of batch k+1 is issued on a side stream while step k runs; ``get`` makes the
    compute stream wait on that copy's event.
    """

    def __init__(self, source, batch: int, seq: int, device: torch.device, depth: int = 2):
        self.source, self.batch, self.seq, self.device = source, batch, seq, device
        self.depth = depth
        self.host = [(torch.empty((batch, seq), dtype=torch.int32, pin_memory=True),
                      torch.empty((batch, seq), dtype=torch.int32, pin_memory=True)) for _ in range(depth + 1)]
        self.dev = [(torch.empty((batch, seq), dtype=torch.int32, device=device),
                     torch.empty((batch, seq), dtype=torch.int32, device=device)) for _ in range(depth + 1)]
        self.copy_stream = torch.cuda.Stream(device=device)
        self.events = [torch.cuda.Event() for _ in range(depth + 1)]
        self.free: Queue = Queue()
        self.ready: Queue = Queue()
        for i in range(depth + 1):
            self.free.put(i)
        self.h2d_bytes = 2 * batch * seq * 4
        self._stop = False
        self._error: BaseException | None = None
        self.thread = threading.Thread(target=self._fill, daemon=True)
        self.thread.start()
        self._inflight: list[int] = []

    def _fill(self):
        try:
            while not self._stop:
                i = self.free.get()
                if i is None:
                    return
                hx, hy = self.host[i]
                if hasattr(self.source, "next_into"):
                    self.source.next_into(hx, hy, self.batch, self.seq)
                else:
                    x, y = self.source.next(self.batch, self.seq)
                    hx.numpy()[...] = x
                    hy.numpy()[...] = y
                self.ready.put(i)
        except BaseException as e:  # handed to the consumer, which would otherwise wait forever
            self._error = e
            self.ready.put(-1)

    def get(self):
        if self._error is not None:  # every later call raises too, instead of waiting on an empty queue
            raise RuntimeError(f"the data thread failed: {self._error!r}") from self._error
        i = self.ready.get()
        if i < 0:
            self.ready.put(-1)
            raise RuntimeError(f"the data thread failed: {self._error!r}") from self._error
        hx, hy = self.host[i]
        dx, dy = self.dev[i]
        cur = torch.cuda.current_stream(self.device)
        # the device slot may still be read by an earlier step
        self.copy_stream.wait_stream(cur)
        with torch.cuda.stream(self.copy_stream):
            dx.copy_(hx, non_blocking=True)
            dy.copy_(hy, non_blocking=True)
            self.events[i].record(self.copy_stream)
        cur.wait_event(self.events[i])
        self._inflight.append(i)
        if len(self._inflight) > 1:  # the host slot of the previous batch is free once its copy completed
            j = self._inflight.pop(0)
            self.events[j].synchronize()
            self.free.put(j)
        return dx, dy

    def close(self):
        self._stop = True
        self.free.put(None)
