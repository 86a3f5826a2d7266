"""Fused optimizer step for :class:`~bitresearch_b200.optim.muon_adamw.MuonAdamW` on sm_100a.

AdamW: one multi-tensor launch over every AdamW parameter of the shard (fp32 master, moments, optional
bf16 shadow). Muon, per stack of equally shaped matrices: momentum + normalisation kernel -> five
batched Polar-Express iterations on tcgen05 GEMMs (bf16 operands, fp32 accumulation, the ``b*A + c*A@A``
and ``a*X + X@B`` combinations fused into GEMM epilogues) -> NorMuon + cautious-decay update kernel.
Matrices too small for 16-byte TMA rows (the [32, KV] value-embedding gates) take the eager path.
"""
from __future__ import annotations

import math

import torch

from ..optim.muon_adamw import POLAR_EXPRESS_COEFFS, normuon_scale, polar_express
from . import gemm
from ._ext import ext

_MAX_ADAM = 32


def step_adamw(opt, grads, skip: torch.Tensor | None = None) -> None:
    """``skip``: optional int32 [1] device word; when it holds nonzero at run time the kernels leave
    parameters and state unchanged (the device-side agreement of a data-parallel step)."""
    P, G, Ms, Vs, Sh, H = [], [], [], [], [], []
    for group, lr, (b1, b2) in opt.adam_groups:
        for n in opt.groups[group]:
            g = grads.get(n)
            if g is None:
                continue
            st = opt.state[n]
            st["step"] += 1
            t = st["step"]
            P.append(opt.params[n].data)
            G.append(g.contiguous())
            Ms.append(st["m"])
            Vs.append(st["v"])
            sh = opt.shadows.get(n)
            Sh.append(sh if sh is not None and sh.is_contiguous() else torch.Tensor())
            H += [lr * opt.lr_multiplier, b1, b2, 1 - b1 ** t, 1 - b2 ** t, 1e-10, 0.0]
    E = ext()
    for i in range(0, len(P), _MAX_ADAM):
        j = i + _MAX_ADAM
        E.adamw_multi(P[i:j], G[i:j], Ms[i:j], Vs[i:j], Sh[i:j], H[7 * i:7 * j], skip)
    for k, n in enumerate([n for g, _, _ in opt.adam_groups for n in opt.groups[g] if n in grads]):
        sh = opt.shadows.get(n)
        if sh is not None and not sh.is_contiguous():
            sh.copy_(opt.params[n])


def _gemm_ok(r: int, c: int) -> bool:
    return min(r, c) >= 64 and r % 8 == 0 and c % 8 == 0


def polar_express_tc(X: torch.Tensor, steps: int, bufs: dict) -> torch.Tensor:
    """Batched Polar-Express on tcgen05 GEMMs; ``X`` bf16 [S, r, c], already normalised."""
    S, r, c = X.shape
    small = min(r, c)
    key = (S, r, c)
    if key not in bufs:
        dev = X.device
        bufs[key] = (torch.empty(S, small, small, dtype=torch.bfloat16, device=dev),
                     torch.empty(S, small, small, dtype=torch.bfloat16, device=dev),
                     torch.empty(S, r, c, dtype=torch.bfloat16, device=dev))
    A, Bm, Y = bufs[key]
    cur, nxt = X, Y
    for a, b, cc in POLAR_EXPRESS_COEFFS[: min(steps, len(POLAR_EXPRESS_COEFFS))]:
        if r >= c:
            gemm.matmul(cur.mT, cur, out=A)                                   # A = X^T X
            gemm.matmul(A, A, out=Bm, aux=A, alpha=cc, beta=b)                # B = b A + c A A
            gemm.matmul(cur, Bm, out=nxt, aux=cur, alpha=1.0, beta=a)         # X = a X + X B
        else:
            gemm.matmul(cur, cur.mT, out=A)                                   # A = X X^T
            gemm.matmul(A, A, out=Bm, aux=A, alpha=cc, beta=b)
            gemm.matmul(Bm, cur, out=nxt, aux=cur, alpha=1.0, beta=a)         # X = a X + B X
        cur, nxt = nxt, cur
    return cur


def step_muon(opt, grads, skip: torch.Tensor | None = None) -> None:
    mu = opt.muon_momentum
    wd = opt.muon_weight_decay
    E = ext()
    if not hasattr(opt, "_ws"):
        opt._ws = {}
    for shape, names in opt.stacks.items():
        names = [n for n in names if n in grads and grads[n] is not None]
        if not names:
            continue
        r, c = shape
        lr = opt.matrix_lr * opt.lr_multiplier * max(1.0, math.sqrt(max(r / c, c / r)))
        if not _gemm_ok(r, c):
            _muon_eager(opt, names, grads, mu, lr, wd, skip)
            continue
        for i in range(0, len(names), 64):
            chunk = names[i:i + 64]
            S = len(chunk)
            key = ("x", S, r, c)
            if key not in opt._ws:
                dev = grads[chunk[0]].device
                opt._ws[key] = (torch.empty(S, r, c, dtype=torch.bfloat16, device=dev),
                                torch.empty(E.muon_prepare_scratch(S, r * c), dtype=torch.float32, device=dev),
                                torch.empty(E.muon_finish_scratch(S, r, c), dtype=torch.float32, device=dev))
            X, ss, work = opt._ws[key]
            G = [grads[n].contiguous() for n in chunk]
            E.muon_prepare(G, [opt.state[n]["mom"] for n in chunk], mu, X, ss, skip)
            Xo = polar_express_tc(X, opt.ns_steps, opt._ws)
            sh = [opt.shadows.get(n, torch.Tensor()) for n in chunk]
            E.muon_finish(Xo, G, [opt.params[n].data for n in chunk], [opt.state[n]["sec"] for n in chunk], sh,
                          r, c, opt.beta2, lr, wd, work, skip)
            for n in chunk:
                opt.state[n]["step"] += 1


def _muon_eager(opt, names, grads, mu, lr, wd, skip=None) -> None:
    G = torch.stack([grads[n].float() for n in names])
    P = torch.stack([opt.params[n].float() for n in names])
    M = torch.stack([opt.state[n]["mom"] for n in names])
    Sc = torch.stack([opt.state[n]["sec"] for n in names])
    P0, M0, Sc0 = P.clone(), M.clone(), Sc.clone()
    M.mul_(mu).add_(G, alpha=1 - mu)
    X = polar_express(G * (1 - mu) + M * mu, opt.ns_steps, torch.float32)
    X, Sc = normuon_scale(X, Sc, opt.beta2)
    mask = (G * P >= 0).to(P.dtype)
    P.sub_(lr * X + lr * wd * P * mask)
    if skip is not None:  # device-side select: the old values where the step is skipped
        keep = skip.bool()
        P, M, Sc = torch.where(keep, P0, P), torch.where(keep, M0, M), torch.where(keep, Sc0, Sc)
    for j, n in enumerate(names):
        opt.params[n].data.copy_(P[j])
        opt.state[n]["mom"].copy_(M[j])
        opt.state[n]["sec"].copy_(Sc[j])
        opt.state[n]["step"] += 1
        if n in opt.shadows:
            opt.shadows[n].copy_(P[j])
