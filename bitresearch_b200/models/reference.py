"""Plain fp32 PyTorch oracle of the reference GPT forward pass.

This restates the reference's CPU parity model (scripts/export_reference.py:83-244), which is
itself a line-by-line restatement of the trainer's model (src/model/gpt.ts:183-325). Two places
where the two reference files disagree are switchable:

* ``gate_from_prenorm``: the value-embedding gate reads the *un-normalised* ladder output in
  gpt.ts:230 and the normalised ``pre_norm`` in export_reference.py:195. Default: gpt.ts.
* ``exporter_window``: gpt.ts keeps ``ws`` keys including self (gpt.ts:264-271); the exporter keeps
  ``ws + 1`` (export_reference.py:53-61). Default: gpt.ts.

The oracle is intentionally op-by-op and materialises the full [B,H,T,T] scores, exactly like the
reference, so it is only meant for small shapes.
"""
from __future__ import annotations

import math
from typing import Mapping

import torch
import torch.nn.functional as F

from ..config import VE_GATE_CHANNELS, GPTConfig, compute_window_sizes, has_value_embedding


def rms_norm(x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)


def rope_tables(seq_len: int, head_dim: int, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    t = torch.arange(0, seq_len, dtype=torch.float32, device=device)
    freqs = torch.outer(t, inv_freq)
    return torch.cos(freqs), torch.sin(freqs)


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    _, t, _, hd = x.shape
    h = hd // 2
    x1, x2 = x[..., :h], x[..., h:]
    c = cos[:t].view(1, t, 1, h)
    s = sin[:t].view(1, t, 1, h)
    return torch.cat([x1 * c + x2 * s, x1 * (-s) + x2 * c], dim=-1)


def attention_mask(seq_len: int, window: int, exporter_window: bool = False, device=None) -> torch.Tensor:
    """Additive mask: causal -1e9 plus window -1e9 (gpt.ts:200, 260-271)."""
    i = torch.arange(seq_len, device=device).view(seq_len, 1)
    j = torch.arange(seq_len, device=device).view(1, seq_len)
    mask = torch.where(j <= i, 0.0, -1e9)
    if exporter_window:
        allowed = (j <= i) & (j >= i - window)
        return torch.where(allowed, 0.0, -1e9)
    if 0 < window < seq_len:
        lo = torch.clamp(i - (window - 1), min=0)
        mask = mask - torch.where(j < lo, 1e9, 0.0)
    return mask


def reference_forward(
    params: Mapping[str, torch.Tensor],
    cfg: GPTConfig,
    idx: torch.Tensor,
    targets: torch.Tensor | None = None,
    *,
    gate_from_prenorm: bool = False,
    exporter_window: bool = False,
    reduction: str = "mean",
):
    """Returns (logits [B,T,V], loss) with the reference's CE (log(softmax+1e-10), mean over B*T)."""
    B, T = idx.shape
    H, KV, hd, D = cfg.n_head, cfg.n_kv_head, cfg.head_dim, cfg.n_embd
    g = H // KV
    windows = compute_window_sizes(cfg)
    cos, sin = rope_tables(cfg.sequence_len, hd, idx.device)

    x = rms_norm(params["wte"][idx])
    x0 = x
    cur = x
    for i in range(cfg.n_layer):
        cur = cur * params["residLambdas"][i] + x0 * params["x0Lambdas"][i]
        pre = rms_norm(cur)
        flat = pre.reshape(B * T, D)
        q = (flat @ params[f"layer{i}_q"]).view(B, T, H, hd)
        k = (flat @ params[f"layer{i}_k"]).view(B, T, KV, hd)
        v = (flat @ params[f"layer{i}_v"]).view(B, T, KV, hd)
        if has_value_embedding(i, cfg.n_layer):
            ve = params[f"ve_{i}"][idx].view(B, T, KV, hd)
            gin = (pre if gate_from_prenorm else cur)[..., :VE_GATE_CHANNELS].reshape(B * T, VE_GATE_CHANNELS)
            gate = 2.0 * torch.sigmoid(gin @ params[f"layer{i}_ve_gate"]).view(B, T, KV, 1)
            v = v + ve * gate
        q = rms_norm(apply_rotary(q, cos, sin))
        k = rms_norm(apply_rotary(k, cos, sin))
        if g > 1:
            k = k.unsqueeze(3).expand(B, T, KV, g, hd).reshape(B, T, H, hd)
            v = v.unsqueeze(3).expand(B, T, KV, g, hd).reshape(B, T, H, hd)
        q, k, v = (t.permute(0, 2, 1, 3) for t in (q, k, v))
        scores = (q @ k.transpose(-2, -1)) / math.sqrt(hd)
        scores = scores + attention_mask(T, windows[i][0], exporter_window, idx.device).view(1, 1, T, T)
        probs = F.softmax(scores, dim=-1)
        o = (probs @ v).permute(0, 2, 1, 3).reshape(B * T, D)
        cur = cur + (o @ params[f"layer{i}_proj"]).view(B, T, D)
        h = F.relu(rms_norm(cur).reshape(B * T, D) @ params[f"layer{i}_fc"]).square()
        cur = cur + (h @ params[f"layer{i}_mlp_proj"]).view(B, T, D)

    xf = rms_norm(cur).reshape(B * T, D)
    logits = xf @ params["lmHead"].t()
    logits = torch.tanh(logits / 15.0) * 15.0
    if targets is None:
        return logits.view(B, T, -1), None
    flat_t = targets.reshape(-1)
    logp = torch.log(F.softmax(logits, dim=-1) + 1e-10)
    nll = -logp.gather(1, torch.relu(flat_t).long().unsqueeze(1)).squeeze(1)
    valid = (flat_t != -1).to(nll.dtype)
    if reduction == "none":
        return logits.view(B, T, -1), nll.view(B, T)
    return logits.view(B, T, -1), (nll * valid).mean()
