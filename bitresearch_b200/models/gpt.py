"""The autoresearch GPT with the reference trainer's parameter names and semantics.

Parameter names, shapes and flat order follow src/model/gpt.ts:88-128 and 330-342 so that
checkpoints are interchangeable with the reference's ``.safetensors`` files:

  wte [V,D], lmHead [V,D] (used as x @ lmHead^T), residLambdas [L], x0Lambdas [L],
  layer{i}_{q,k,v,proj,fc,mlp_proj} stored [in, out] (x @ W), layer{i}_ve_gate [32, KV],
  ve_{i} [V, KV*hd] on value-embedding layers.

``forward_torch`` is the eager PyTorch path (autograd, any device/dtype). The sm_100a path is the
hand-scheduled engine in :mod:`bitresearch_b200.models.engine`, which shares this module's
parameters.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import (VE_GATE_CHANNELS, GPTConfig, compute_window_sizes, effective_window,
                      estimate_flops_per_token, has_value_embedding)


def param_specs(cfg: GPTConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, group) in the reference's flat order (gpt.ts:330-342).

    group is one of lmHead, wte, valueEmbeds, residLambdas, x0Lambdas, matrices (muon.ts:238-290).
    """
    V, D, L, KV = cfg.vocab_size, cfg.n_embd, cfg.n_layer, cfg.kv_dim
    specs = [("wte", (V, D), "wte"), ("lmHead", (V, D), "lmHead"),
             ("residLambdas", (L,), "residLambdas"), ("x0Lambdas", (L,), "x0Lambdas")]
    for i in range(L):
        specs += [
            (f"layer{i}_q", (D, cfg.n_head * cfg.head_dim), "matrices"),
            (f"layer{i}_k", (D, KV), "matrices"),
            (f"layer{i}_v", (D, KV), "matrices"),
            (f"layer{i}_proj", (D, D), "matrices"),
            (f"layer{i}_fc", (D, 4 * D), "matrices"),
            (f"layer{i}_mlp_proj", (4 * D, D), "matrices"),
        ]
        if has_value_embedding(i, L):
            specs.append((f"layer{i}_ve_gate", (VE_GATE_CHANNELS, cfg.n_kv_head), "matrices"))
    for i in range(L):
        if has_value_embedding(i, L):
            specs.append((f"ve_{i}", (V, KV), "valueEmbeds"))
    return specs


class GPT(nn.Module):
    def __init__(self, cfg: GPTConfig, init: str = "karpathy", seed: int = 42, device=None):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        self.window_sizes = compute_window_sizes(cfg)
        self.specs = param_specs(cfg)
        self.params = nn.ParameterDict()
        for name, shape, _ in self.specs:
            self.params[name] = nn.Parameter(torch.empty(shape, dtype=torch.float32, device=device))
        self.init_weights(init, seed)
        self.compute_dtype: torch.dtype | None = None  # matmul operand dtype of the eager path
        self.attn_impl = "sdpa"  # eager attention: "sdpa" or "flex" (fused sliding window, under torch.compile)
        cos, sin = _rope(cfg.sequence_len, cfg.head_dim, device)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def init_weights(self, init: str = "karpathy", seed: int = 42) -> None:
        """``karpathy``: the trainer's init (gpt.ts:79-128). ``normal``: N(0, 0.02) of the parity
        oracle (export_reference.py:136-152)."""
        gen = torch.Generator(device="cpu").manual_seed(seed)
        D = self.cfg.n_embd
        s = math.sqrt(3.0) * D ** -0.5
        for name, shape, group in self.specs:
            p = self.params[name]
            if name == "residLambdas":
                t = torch.ones(shape)
            elif name == "x0Lambdas":
                t = torch.full(shape, 0.1)
            elif name.endswith("_proj") or name.endswith("_ve_gate"):
                t = torch.zeros(shape)  # proj, mlp_proj, ve_gate start at zero in both inits
            elif init == "normal":
                t = torch.randn(shape, generator=gen) * 0.02
            elif name == "wte":
                t = torch.randn(shape, generator=gen)
            elif name == "lmHead":
                t = torch.randn(shape, generator=gen) * 0.001
            else:  # q, k, v, fc, ve_*
                t = (torch.rand(shape, generator=gen) * 2 - 1) * s
            p.copy_(t.to(p.device))

    # ------------------------------------------------------------------ helpers
    def named(self) -> dict[str, torch.Tensor]:
        return {n: self.params[n] for n, _, _ in self.specs}

    def ordered_params(self) -> list[nn.Parameter]:
        return [self.params[n] for n, _, _ in self.specs]

    def num_params(self) -> int:
        return sum(p.numel() for p in self.params.values())

    def param_groups(self) -> dict[str, list[str]]:
        groups: dict[str, list[str]] = {}
        for n, _, g in self.specs:
            groups.setdefault(g, []).append(n)
        return groups

    def estimate_flops_per_token(self) -> int:
        return estimate_flops_per_token(self.cfg)

    # ------------------------------------------------------------------ eager forward
    def forward(self, idx, targets=None, reduction: str = "mean", exact_ce: bool = True):
        return self.forward_torch(idx, targets, reduction=reduction, exact_ce=exact_ce,
                                  compute_dtype=self.compute_dtype)

    def forward_torch(self, idx: torch.Tensor, targets: torch.Tensor | None = None, reduction: str = "mean",
                      exact_ce: bool = True, compute_dtype: torch.dtype | None = None):
        """Eager forward. Returns the mean loss (``reduction='mean'``), per-token nats [B,T] with 0 at
        ignored (-1) targets (``'none'``) or logits (``targets is None``).

        ``exact_ce`` uses the reference's ``-log(softmax + 1e-10)`` (gpt.ts:306-313); otherwise
        ``F.cross_entropy``. ``compute_dtype`` casts matmul operands (bf16 for the GPU baseline).
        """
        cfg = self.cfg
        P = self.params
        B, T = idx.shape
        H, KV, hd, D = cfg.n_head, cfg.n_kv_head, cfg.head_dim, cfg.n_embd
        cd = compute_dtype

        def mm(a, w):
            if cd is None:
                return a @ w
            return (a.to(cd) @ w.to(cd)).float()

        x = _rms(P["wte"][idx])
        x0 = x
        cur = x
        cos = self.rope_cos[:T]
        sin = self.rope_sin[:T]
        for i in range(cfg.n_layer):
            cur = cur * P["residLambdas"][i] + x0 * P["x0Lambdas"][i]
            pre = _rms(cur).reshape(B * T, D)
            q = mm(pre, P[f"layer{i}_q"]).view(B, T, H, hd)
            k = mm(pre, P[f"layer{i}_k"]).view(B, T, KV, hd)
            v = mm(pre, P[f"layer{i}_v"]).view(B, T, KV, hd)
            if has_value_embedding(i, cfg.n_layer):
                gin = cur[..., :VE_GATE_CHANNELS].reshape(B * T, VE_GATE_CHANNELS)  # gpt.ts:230 semantics
                gate = 2.0 * torch.sigmoid(gin @ P[f"layer{i}_ve_gate"]).view(B, T, KV, 1)
                v = v + P[f"ve_{i}"][idx].view(B, T, KV, hd) * gate
            q = _rms(_rotary(q, cos, sin))
            k = _rms(_rotary(k, cos, sin))
            o = _attention(q, k, v, effective_window(self.window_sizes[i][0], T), cd, self.attn_impl)
            cur = cur + mm(o.reshape(B * T, D), P[f"layer{i}_proj"]).view(B, T, D)
            h = F.relu(mm(_rms(cur).reshape(B * T, D), P[f"layer{i}_fc"])).square()
            cur = cur + mm(h, P[f"layer{i}_mlp_proj"]).view(B, T, D)
        xf = _rms(cur).reshape(B * T, D)
        logits = mm(xf, P["lmHead"].t())
        logits = torch.tanh(logits / 15.0) * 15.0
        if targets is None:
            return logits.view(B, T, -1)
        flat_t = targets.reshape(-1).long()
        if exact_ce:
            logp = torch.log(torch.softmax(logits, -1) + 1e-10)
            nll = -logp.gather(1, flat_t.clamp(min=0).unsqueeze(1)).squeeze(1)
        else:
            nll = F.cross_entropy(logits, flat_t.clamp(min=0), reduction="none")
        valid = (flat_t != -1).to(nll.dtype)
        if reduction == "none":  # the reference's masked per-token loss: 0 at ignored positions
            return (nll * valid).view(B, T)
        return (nll * valid).sum() / nll.numel()


def _rope(seq_len: int, head_dim: int, device=None):
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    freqs = torch.outer(torch.arange(seq_len, dtype=torch.float32), inv_freq)
    return torch.cos(freqs).to(device), torch.sin(freqs).to(device)


def _rms(x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    x32 = x.float()
    return x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)


def _rotary(x, cos, sin):
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c = cos.view(1, -1, 1, h)
    s = sin.view(1, -1, 1, h)
    return torch.cat([x1 * c + x2 * s, x2 * c - x1 * s], dim=-1)


_FLEX_MASKS: dict = {}


def _flex_attention(q, k, v, window: int):
    """Sliding-window causal attention through PyTorch's flex attention (a fused kernel that skips blocks
    outside the band), for the baselines; q, k, v [B, H, T, hd]."""
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention
    T = q.shape[2]
    key = (T, window, q.device)
    if key not in _FLEX_MASKS:
        def band(b, h, qi, kj):
            return (kj <= qi) & (kj > qi - window)
        _FLEX_MASKS[key] = create_block_mask(band, B=None, H=None, Q_LEN=T, KV_LEN=T, device=q.device)
    return flex_attention(q, k, v, block_mask=_FLEX_MASKS[key], enable_gqa=k.shape[1] != q.shape[1])


def _attention(q, k, v, window: int, cd, impl: str = "sdpa"):
    """q,k,v [B,T,H|KV,hd]; causal with a ``window``-key band (keys i-window+1..i). ``impl='flex'`` runs
    flex attention (meant to be used under ``torch.compile``) instead of SDPA with a boolean band mask."""
    B, T, H, hd = q.shape
    KV = k.shape[2]
    if impl == "flex":
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
        if cd is not None:
            q, k, v = q.to(cd), k.to(cd), v.to(cd)
        return _flex_attention(q, k, v, window).float().transpose(1, 2)
    if KV != H:
        k = k.repeat_interleave(H // KV, dim=2)
        v = v.repeat_interleave(H // KV, dim=2)
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    if cd is not None:
        q, k, v = q.to(cd), k.to(cd), v.to(cd)
    if window >= T:
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    else:
        i = torch.arange(T, device=q.device).view(T, 1)
        j = torch.arange(T, device=q.device).view(1, T)
        mask = (j <= i) & (j > i - window)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    return o.float().transpose(1, 2)
