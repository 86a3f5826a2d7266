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


def _config_from_checkpoint(path: str, fallback):
    """The TrainConfig stored in a checkpoint's ``trainConfig`` metadata; for a checkpoint written by the
    reference, which stores only the model config (``config``, src/distributed/trainer.ts:1132-1137),
    ``fallback`` with that model."""
    import json

    from . import checkpoint as ckpt
    from .config import GPTConfig, TrainConfig
    _, meta = ckpt.load(path)
    raw = meta.get("trainConfig")
    if raw:
        d = json.loads(raw)
        return TrainConfig.from_dict(json.loads(d) if isinstance(d, str) else d)
    if meta.get("config"):
        fallback.model = GPTConfig.from_reference_dict(json.loads(meta["config"]))
    return fallback


def main(argv=None) -> int:
    """``python -m bitresearch_b200.eval --checkpoint PATH [--preset P] [key=value ...]``: loads a checkpoint
    and prints its ``val_bpb`` on the configured validation split (the reference's load-checkpoint then
    evaluate path, src/distributed/trainer.ts:1225-1289 and :897-976). The training config comes from the
    checkpoint's metadata when it has one, else from ``--preset`` with the checkpoint's model config;
    overrides apply on top (e.g. ``data=... data_path=... eval_tokens=...``)."""
    import argparse
    import sys

    from .config import apply_overrides, preset
    from .train import Trainer
    ap = argparse.ArgumentParser(description="evaluate a checkpoint's bits per byte")
    ap.add_argument("--checkpoint", required=True)
    ap.add_argument("--preset", default="d512")
    ap.add_argument("--device", default=None)
    ap.add_argument("overrides", nargs="*")
    args = ap.parse_args(argv)
    cfg = _config_from_checkpoint(args.checkpoint, preset(args.preset))
    cfg = apply_overrides(cfg, list(args.overrides) + ["results_tsv=", "log_every=0", "status_port=-1"])
    if args.device is None and not torch.cuda.is_available():
        cfg.impl, cfg.dtype = "torch", "fp32"
    tr = Trainer(cfg, device=args.device, log=lambda m: print(m, file=sys.stderr))
    tr.initialize()
    info = tr.load_checkpoint(args.checkpoint)
    bpb = tr.evaluate_bpb()
    tr.destroy()
    print(f"val_bpb:          {bpb:.6f}")
    print(f"step:             {info.get('step', 0)}")
    if "val_bpb_floor" in tr.metrics.extra:
        print(f"val_bpb_floor:    {tr.metrics.extra['val_bpb_floor']:.6f}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
