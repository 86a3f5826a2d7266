"""Bits-per-byte evaluation (Karpathy's ``evaluate_bpb`` semantics).

The reference has two implementations (src/data/dataloader.ts:503-551 and
src/distributed/trainer.ts:897-976). Both sum per-token nats over targets whose byte length is
positive, sum those byte lengths, and report ``nats / (ln 2 * bytes)``; the number of batches is
``floor(eval_tokens / (B*T))``. This module implements that single definition over a held-out split:
tokens with ``token_bytes == 0`` (special tokens) and ignored targets (``-1``) are excluded.

The per-token nats come from the model's ``reduction='none'`` forward; on the sm_100a engine the
fused lm_head/cross-entropy kernel also produces the two byte-masked sums directly.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def bpb_from_sums(total_nats: float, total_bytes: float) -> float:
    if total_bytes <= 0:
        return 0.0
    return total_nats / (math.log(2) * total_bytes)


@torch.no_grad()
def evaluate_bpb(per_token_nats_fn, batch_source, token_bytes: np.ndarray, batch: int, seq: int,
                 eval_tokens: int, device="cpu") -> tuple[float, float, float]:
    """Returns (bpb, total_nats, total_bytes).

    ``per_token_nats_fn(inputs, targets) -> nats [B,T]`` (tensor); ``batch_source.next(B,T)``
    yields host int32 arrays.
    """
    steps = max(1, eval_tokens // (batch * seq))
    tb = torch.as_tensor(np.asarray(token_bytes, dtype=np.int64), device=device)
    total_nats = torch.zeros((), dtype=torch.float64, device=device)
    total_bytes = torch.zeros((), dtype=torch.float64, device=device)
    for _ in range(steps):
        x, y = batch_source.next(batch, seq)
        x = torch.as_tensor(np.ascontiguousarray(x), device=device)
        y = torch.as_tensor(np.ascontiguousarray(y), device=device)
        nats = per_token_nats_fn(x, y).reshape(-1).double()
        yf = y.reshape(-1).long()
        nbytes = torch.where(yf >= 0, tb[yf.clamp(min=0)], torch.zeros_like(yf))
        m = nbytes > 0
        total_nats += torch.where(m, nats, torch.zeros_like(nats)).sum()
        total_bytes += nbytes.sum().double()
    n, b = float(total_nats), float(total_bytes)
    return bpb_from_sums(n, b), n, b
