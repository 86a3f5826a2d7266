"""Top-k gradient sparsification with error feedback (Deep Gradient Compression).

Semantics follow src/distributed/gradient-sparsifier.ts:

* the first ``warmup_steps`` calls are dense (gradient-sparsifier.ts:65-67, 87-91);
* ``g += e`` (error feedback), then optional momentum correction ``v = mu*v + g; g = v``
  (gradient-sparsifier.ts:103-118);
* threshold = the ``floor(S*(1-k))``-th smallest of ``S`` sampled ``|g|`` values
  (gradient-sparsifier.ts:211-227); entries with ``|g| >= thr`` are kept and their residual cleared,
  the rest go to the residual and are zeroed (gradient-sparsifier.ts:124-137);
* wire codec ``[length u32 | count u32 | indices u32[] | values f32[]]`` (gradient-sparsifier.ts:161-193).

With momentum the reference's residual is the whole velocity and the velocity is never cleared, so an
entry that stays below the threshold grows as ``e <- (1 + mu) e + g`` (1.9x per step at mu = 0.9).
``momentum_masking=True`` runs Deep Gradient Compression as published instead (Lin et al., 2018):
``u = mu u + g``, ``v = v + u``, send the top-k of ``v``, clear ``v`` and ``u`` where sent. The default
keeps the reference's update.

``GradientSparsifier`` is the torch implementation (any device). On B200 the same math runs fused in
one kernel pass (threshold from a device-side sample, select, EF update, compaction to an
index/f16-value payload) in :mod:`bitresearch_b200.parallel.comm`, and this class is its oracle.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class SparseGradient:
    length: int
    indices: torch.Tensor  # int64
    values: torch.Tensor   # float32


class GradientSparsifier:
    def __init__(self, top_k_ratio: float = 0.10, warmup_steps: int = 100, sample_size: int = 10000,
                 momentum_factor: float = 0.9, seed: int = 0, momentum_masking: bool = False):
        if not (0 < top_k_ratio <= 1):
            raise ValueError(f"topKRatio must be in (0, 1], got {top_k_ratio}")
        self.k = top_k_ratio
        self.warmup_steps = warmup_steps
        self.sample_size = sample_size
        self.mu = momentum_factor
        self.masking = momentum_masking
        self.error: torch.Tensor | None = None
        self.velocity: torch.Tensor | None = None
        self.step = 0
        self.gen = torch.Generator().manual_seed(seed)

    def reset(self):
        self.error = None
        self.velocity = None
        self.step = 0

    @property
    def is_dense_step(self) -> bool:
        return self.step < self.warmup_steps

    def find_threshold(self, g: torch.Tensor) -> float:
        N = g.numel()
        S = min(N, self.sample_size)
        idx = torch.randint(0, N, (S,), generator=self.gen).to(g.device)
        samples = g.reshape(-1)[idx].abs().sort().values
        cut = math.floor(S * (1.0 - self.k))
        return float(samples[min(cut, S - 1)])

    @torch.no_grad()
    def sparsify(self, g: torch.Tensor) -> SparseGradient:
        """Sparsify ``g`` (flat fp32) in place; returns the kept entries."""
        N = g.numel()
        self.step += 1
        if self.is_dense_step:
            return SparseGradient(N, torch.arange(N, device=g.device), g.clone())
        if self.error is None or self.error.numel() != N:
            self.error = torch.zeros_like(g)
        if self.mu > 0 and (self.velocity is None or self.velocity.numel() != N):
            self.velocity = torch.zeros_like(g)
        if self.masking and self.velocity is not None and self.mu > 0:
            self.velocity.mul_(self.mu).add_(g)  # u = m u + g
            g.copy_(self.error).add_(self.velocity)  # v = v + u
        else:
            g.add_(self.error)
            if self.velocity is not None and self.mu > 0:
                self.velocity.mul_(self.mu).add_(g)
                g.copy_(self.velocity)
        thr = self.find_threshold(g)
        keep = g.abs() >= thr
        self.error.copy_(torch.where(keep, torch.zeros_like(g), g))
        if self.masking and self.velocity is not None and self.mu > 0:
            self.velocity.mul_(~keep)
        g.mul_(keep)
        idx = keep.nonzero().squeeze(1)
        return SparseGradient(N, idx, g[idx].clone())

    @staticmethod
    def densify(sp: SparseGradient) -> torch.Tensor:
        out = torch.zeros(sp.length, dtype=torch.float32, device=sp.values.device)
        out[sp.indices] = sp.values.float()
        return out

    @staticmethod
    def encode(sp: SparseGradient) -> bytes:
        n = sp.indices.numel()
        return (struct.pack("<II", sp.length, n) + sp.indices.cpu().numpy().astype("<u4").tobytes()
                + sp.values.cpu().float().numpy().astype("<f4").tobytes())

    @staticmethod
    def decode(buf: bytes) -> SparseGradient:
        length, n = struct.unpack("<II", buf[:8])
        idx = np.frombuffer(buf, dtype="<u4", count=n, offset=8).astype(np.int64)
        val = np.frombuffer(buf, dtype="<f4", count=n, offset=8 + 4 * n).copy()
        return SparseGradient(length, torch.from_numpy(idx), torch.from_numpy(val))

    @staticmethod
    def compression_ratio(sp: SparseGradient) -> float:
        return (8 + sp.indices.numel() * 8) / (sp.length * 4)
