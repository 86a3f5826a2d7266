"""Plain PyTorch data-parallel baselines of the same GPT: DistributedDataParallel (NCCL bucketed
all-reduce overlapped with backward), cuBLAS bf16 matmuls, ``F.cross_entropy`` and the eager MuonAdamW
(bf16 Newton-Schulz), replicated on every rank. No kernel of this repository runs on these paths.

* ``compile=False``: eager, ``scaled_dot_product_attention`` (a boolean band mask on the sliding-window
  layers, which keeps SDPA off its flash kernel there).
* ``compile=True``: the model under ``torch.compile`` with flex attention, a fused sliding-window kernel
  that skips the blocks outside the band on every layer: the strongest stock-PyTorch form of the model.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP

from bitresearch_b200.config import TrainConfig
from bitresearch_b200.models.gpt import GPT
from bitresearch_b200.optim.muon_adamw import MuonAdamW


class DDPBaseline:
    def __init__(self, cfg: TrainConfig, device: torch.device, compile: bool = False):
        self.cfg = cfg
        self.device = device
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.model = GPT(cfg.model, init="karpathy", seed=42, device=device)
        self.model.compute_dtype = torch.bfloat16
        if compile:
            self.model.attn_impl = "flex"
        self.net = DDP(self.model, device_ids=[device.index]) if self.world > 1 else self.model
        if compile:
            self.net = torch.compile(self.net)
        self.opt = MuonAdamW(self.model.named(), self.model.param_groups(), model_dim=cfg.model.n_embd,
                             ns_dtype="bf16", impl="torch")
        self.opt.lr_multiplier, self.opt.muon_momentum, self.opt.muon_weight_decay = 1.0, 0.95, cfg.weight_decay
        T = cfg.model.sequence_len
        rows = cfg.total_batch_tokens // self.world // T
        self.device_batch = min(cfg.device_batch, rows)
        self.grad_accum = rows // self.device_batch

    def train_step(self, batches) -> torch.Tensor:
        losses = []
        for i, (x, y) in enumerate(batches):
            last = i == len(batches) - 1
            ctx = self.net.no_sync() if (self.world > 1 and not last) else _null()
            with ctx:
                loss = self.net(x, y, exact_ce=False)
                (loss / len(batches)).backward()
            losses.append(loss.detach())
        grads = {n: p.grad for n, p in self.model.named().items()}
        self.opt.step(grads)
        for p in self.model.parameters():
            p.grad = None
        return torch.stack(losses).mean()


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False
