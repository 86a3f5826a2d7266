"""MuonAdamW: Muon (Polar-Express Newton-Schulz + NorMuon + cautious weight decay) for matrices,
AdamW for embeddings, lm_head, value embeddings and the two scalar vectors.

Behaviour follows src/train/muon.ts:

* six parameter groups, stepped in this order (muon.ts:238-290, 327-335): lmHead, wte,
  valueEmbeds, residLambdas, x0Lambdas (AdamW, eps 1e-10, wd 0), then matrices (Muon).
* AdamW (muon.ts:60-96): decoupled decay, bias-corrected moments, per-parameter step counters.
* Muon (muon.ts:138-196): Nesterov momentum, five Polar-Express steps on the smaller Gram
  matrix (coefficients muon.ts:18-24), NorMuon second-moment EMA (beta2 0.95) with reduction
  over columns when rows >= cols, cautious weight decay on ``raw grad * param >= 0`` and
  ``p -= lr * (g + wd * p * mask)``; per-matrix lr scale ``max(1, sqrt(max(r/c, c/r)))``
  (muon.ts:373-378).

The reference allocates the NorMuon buffer as ``[2, rows, 1]`` (muon.ts:306-310), which cannot be
assigned back to a ``[rows, cols]`` parameter; this implementation keeps the intended per-matrix
``[rows, 1]`` / ``[1, cols]`` buffer.

Execution: parameters are grouped by shape and stepped as stacks (one batched Newton-Schulz chain
per shape). ``impl='cuda'`` runs the fused sm_100a kernels (momentum+normalise, tcgen05 GEMMs for
the Newton-Schulz chain, NorMuon+cautious update, multi-tensor AdamW writing fp32 master and bf16
shadow weights); ``impl='torch'`` is the eager path used on CPU and as the oracle. With ``owned`` set,
only those parameters (this rank's shard) are stepped and hold state.
"""
from __future__ import annotations

import math
from collections import OrderedDict
from typing import Iterable

import torch

POLAR_EXPRESS_COEFFS = [
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
]

ADAMW_GROUPS = ("lmHead", "wte", "valueEmbeds", "residLambdas", "x0Lambdas")


def polar_express(X: torch.Tensor, steps: int = 5, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Batched Polar-Express orthogonalisation of ``X`` [..., r, c] (muon.ts:102-132)."""
    r, c = X.shape[-2:]
    X = X.float()
    X = X / (X.norm(dim=(-2, -1), keepdim=True) * 1.02 + 1e-6)
    X = X.to(dtype)
    for a, b, cc in POLAR_EXPRESS_COEFFS[: min(steps, len(POLAR_EXPRESS_COEFFS))]:
        if r >= c:
            A = X.mT @ X
            Bm = b * A + cc * (A @ A)
            X = a * X + X @ Bm
        else:
            A = X @ X.mT
            Bm = b * A + cc * (A @ A)
            X = a * X + Bm @ X
    return X.float()


def normuon_scale(g: torch.Tensor, sec: torch.Tensor, beta2: float) -> tuple[torch.Tensor, torch.Tensor]:
    """NorMuon variance reduction (muon.ts:158-181). g [S,r,c], sec [S,r,1] or [S,1,c]."""
    r, c = g.shape[-2:]
    red_dim = -1 if r >= c else -2
    red_size = c if r >= c else r
    v_mean = g.square().mean(dim=red_dim, keepdim=True)
    v_norm = (v_mean.sum(dim=(-2, -1), keepdim=True) * red_size).sqrt()
    new_sec = sec * beta2 + v_mean * (1 - beta2)
    step_size = (new_sec + 1e-10).rsqrt()
    v_norm_new = (v_mean * red_size * step_size.square()).sum(dim=(-2, -1), keepdim=True).sqrt()
    final = step_size * (v_norm / (v_norm_new + 1e-10))
    return g * final, new_sec


class MuonAdamW:
    def __init__(self, params: "OrderedDict[str, torch.Tensor]", groups: dict[str, list[str]], *,
                 model_dim: int, unembedding_lr=0.004, embedding_lr=0.6, matrix_lr=0.04, scalar_lr=0.5,
                 weight_decay=0.2, adam_betas=(0.8, 0.95), ns_steps=5, beta2=0.95, ns_dtype="fp32",
                 owned: Iterable[str] | None = None, impl: str = "torch", shadows: dict | None = None):
        self.params = params
        self.owned = set(params) if owned is None else set(owned)
        self.impl = impl
        self.ns_steps = ns_steps
        self.beta2 = beta2
        self.ns_dtype = torch.bfloat16 if ns_dtype == "bf16" else torch.float32
        self.shadows = shadows or {}  # name -> bf16 copy refreshed after each step (cuda engine)
        s = (model_dim / 768) ** -0.5
        b = tuple(adam_betas)
        # (group, lr, betas) in the reference's order (muon.ts:238-280)
        self.adam_groups = [
            ("lmHead", unembedding_lr * s, b),
            ("wte", embedding_lr * s, b),
            ("valueEmbeds", embedding_lr * s, b),
            ("residLambdas", scalar_lr * 0.01, b),
            ("x0Lambdas", scalar_lr, (0.96, 0.95)),
        ]
        self.matrix_lr = matrix_lr
        self.weight_decay = weight_decay
        self.groups = {g: [n for n in groups.get(g, []) if n in self.owned] for g in (*ADAMW_GROUPS, "matrices")}
        self.lr_multiplier = 1.0
        self.muon_momentum = 0.95
        self.muon_weight_decay = 0.0
        self.state: dict[str, dict] = {}
        for g in ADAMW_GROUPS:
            for n in self.groups[g]:
                p = params[n]
                self.state[n] = {"step": 0, "m": torch.zeros_like(p, dtype=torch.float32),
                                 "v": torch.zeros_like(p, dtype=torch.float32)}
        # matrices stacked by shape: one Newton-Schulz chain per stack
        self.stacks: "OrderedDict[tuple[int, int], list[str]]" = OrderedDict()
        for n in self.groups["matrices"]:
            self.stacks.setdefault(tuple(params[n].shape), []).append(n)
        for n in self.groups["matrices"]:
            p = params[n]
            r, c = p.shape
            sec_shape = (r, 1) if r >= c else (1, c)
            self.state[n] = {"step": 0, "mom": torch.zeros_like(p, dtype=torch.float32),
                             "sec": torch.zeros(sec_shape, dtype=torch.float32, device=p.device)}

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self, grads: dict[str, torch.Tensor], skip: torch.Tensor | None = None) -> None:
        """``skip`` (fused path only): an int32 [1] device word; nonzero at run time leaves every parameter and
        state tensor unchanged, so a data-parallel step can agree on skipping without a host round trip
        (the host-side step counters still advance; ``undo_steps`` takes them back)."""
        if self.impl == "cuda":
            from ..ops import optim as fused
            fused.step_adamw(self, grads, skip)
            fused.step_muon(self, grads, skip)
            return
        assert skip is None, "a device-side skip needs the fused optimizer"

        for group, lr, (b1, b2) in self.adam_groups:
            for n in self.groups[group]:
                if n not in grads or grads[n] is None:
                    continue
                self._adamw(n, grads[n].float(), lr * self.lr_multiplier, b1, b2, 1e-10, 0.0)
        self._muon_torch(grads)

    def undo_steps(self, names) -> None:
        """Takes back the step counters of ``names`` after a step the device skipped."""
        for n in names:
            if n in self.state and self.state[n].get("step", 0) > 0:
                self.state[n]["step"] -= 1

    def _adamw(self, n, g, lr, b1, b2, eps, wd):
        p = self.params[n]
        st = self.state[n]
        st["step"] += 1
        t = st["step"]
        p.mul_(1 - lr * wd)
        st["m"].mul_(b1).add_(g, alpha=1 - b1)
        st["v"].mul_(b2).addcmul_(g, g, value=1 - b2)
        bias1 = 1 - b1 ** t
        bias2 = 1 - b2 ** t
        denom = (st["v"] / bias2).sqrt().add_(eps)
        p.addcdiv_(st["m"], denom, value=-lr / bias1)
        if n in self.shadows:
            self.shadows[n].copy_(p)

    def _muon_torch(self, grads):
        mu = self.muon_momentum
        wd = self.muon_weight_decay
        for shape, names in self.stacks.items():
            names = [n for n in names if n in grads and grads[n] is not None]
            if not names:
                continue
            r, c = shape
            lr = self.matrix_lr * self.lr_multiplier * max(1.0, math.sqrt(max(r / c, c / r)))
            G = torch.stack([grads[n].float() for n in names])
            P = torch.stack([self.params[n].float() for n in names])
            M = torch.stack([self.state[n]["mom"] for n in names])
            S = torch.stack([self.state[n]["sec"] for n in names])
            M.mul_(mu).add_(G, alpha=1 - mu)
            nest = G * (1 - mu) + M * mu
            X = polar_express(nest, self.ns_steps, self.ns_dtype)
            X, S = normuon_scale(X, S, self.beta2)
            mask = (G * P >= 0).to(P.dtype)
            P.sub_(lr * X + lr * wd * P * mask)
            for j, n in enumerate(names):
                self.params[n].copy_(P[j])
                self.state[n]["mom"].copy_(M[j])
                self.state[n]["sec"].copy_(S[j])
                self.state[n]["step"] += 1
                if n in self.shadows:
                    self.shadows[n].copy_(P[j])

    # ------------------------------------------------------------------ state
    def state_tensors(self) -> "OrderedDict[str, torch.Tensor]":
        """Optimizer state keyed like the reference's ``getState`` (muon.ts:389-402)."""
        out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        for n, st in self.state.items():
            if "m" in st:
                out[f"adam_m_{n}"] = st["m"]
                out[f"adam_v_{n}"] = st["v"]
            else:
                out[f"muon_mom_{n}"] = st["mom"]
                out[f"muon_sec_{n}"] = st["sec"]
        return out

    def state_steps(self) -> dict[str, int]:
        return {n: int(st["step"]) for n, st in self.state.items()}

    def load_state(self, tensors: dict[str, torch.Tensor], steps: dict[str, int]) -> int:
        loaded = 0
        for n, st in self.state.items():
            keys = (("m", f"adam_m_{n}"), ("v", f"adam_v_{n}")) if "m" in st else \
                   (("mom", f"muon_mom_{n}"), ("sec", f"muon_sec_{n}"))
            for k, key in keys:
                if key in tensors:
                    st[k].copy_(tensors[key].to(st[k].device).view_as(st[k]))
                    loaded += 1
            if n in steps:
                st["step"] = int(steps[n])
        return loaded


def lr_multiplier(progress: float, warmup_ratio: float, warmdown_ratio: float, final_lr_frac: float) -> float:
    """trainer.ts:577-589."""
    if progress < warmup_ratio:
        return progress / warmup_ratio if warmup_ratio > 0 else 1.0
    if progress < 1.0 - warmdown_ratio:
        return 1.0
    cooldown = (1.0 - progress) / warmdown_ratio
    return cooldown * 1.0 + (1 - cooldown) * final_lr_frac


def muon_momentum(step: int) -> float:
    """0.85 -> 0.95 over 300 steps (trainer.ts:591-594)."""
    frac = min(step / 300, 1.0)
    return (1 - frac) * 0.85 + frac * 0.95


def weight_decay_at(progress: float, base: float) -> float:
    """trainer.ts:599-601."""
    return base * (1 - progress)
