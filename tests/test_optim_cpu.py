"""MuonAdamW vs a direct per-parameter restatement of src/train/muon.ts in float64."""
import math

import torch

from bitresearch_b200.config import GPTConfig
from bitresearch_b200.models.gpt import GPT
from bitresearch_b200.optim.muon_adamw import (POLAR_EXPRESS_COEFFS, MuonAdamW, lr_multiplier, muon_momentum,
                                               weight_decay_at)


def _ref_polar(X, steps):
    rows, cols = X.shape
    X = X / (X.norm() * 1.02 + 1e-6)
    for a, b, c in POLAR_EXPRESS_COEFFS[:steps]:
        if rows >= cols:
            A = X.t() @ X
            X = a * X + X @ (b * A + c * (A @ A))
        else:
            A = X @ X.t()
            X = a * X + (b * A + c * (A @ A)) @ X
    return X


def _ref_muon(p, g, mom, sec, mu, lr, wd, beta2):
    mom = mom * mu + g * (1 - mu)
    nest = g * (1 - mu) + mom * mu
    x = _ref_polar(nest, 5)
    rows, cols = x.shape
    red = 1 if rows >= cols else 0
    rsize = cols if rows >= cols else rows
    vmean = x.square().mean(red, keepdim=True)
    vnorm = (vmean.sum() * rsize).sqrt()
    sec = sec * beta2 + vmean * (1 - beta2)
    step = (sec + 1e-10).rsqrt()
    vnn = (vmean * rsize * step.square()).sum().sqrt()
    x = x * (step * (vnorm / (vnn + 1e-10)))
    mask = (g * p >= 0).double()
    p = p - (x * lr + p * wd * mask * lr)
    return p, mom, sec


def _ref_adamw(p, g, m, v, t, lr, b1, b2, eps):
    m = m * b1 + g * (1 - b1)
    v = v * b2 + g.square() * (1 - b2)
    denom = (v / (1 - b2 ** t)).sqrt() + eps
    return p - (lr / (1 - b1 ** t)) * m / denom, m, v


def test_muon_adamw_two_steps_match_restatement():
    cfg = GPTConfig(sequence_len=16, vocab_size=64, n_layer=2, n_head=2, n_kv_head=2, n_embd=64)
    model = GPT(cfg, init="normal", seed=3)
    params = model.named()
    ref = {n: p.detach().double().clone() for n, p in params.items()}
    opt = MuonAdamW(params, model.param_groups(), model_dim=cfg.n_embd, ns_dtype="fp32")
    opt.lr_multiplier, opt.muon_momentum, opt.muon_weight_decay = 0.7, 0.9, 0.1
    state = {}
    gen = torch.Generator().manual_seed(5)
    s = (cfg.n_embd / 768) ** -0.5
    glr = {"lmHead": (0.004 * s, (0.8, 0.95)), "wte": (0.6 * s, (0.8, 0.95)), "residLambdas": (0.005, (0.8, 0.95)),
           "x0Lambdas": (0.5, (0.96, 0.95))}
    for t in (1, 2):
        grads = {n: torch.randn(p.shape, generator=gen) * 0.1 for n, p in params.items()}
        opt.step(grads)
        for n, g in grads.items():
            g = g.double()
            p = ref[n]
            if n.startswith("ve_"):
                lr, (b1, b2) = 0.6 * s, (0.8, 0.95)
            elif n in glr:
                lr, (b1, b2) = glr[n]
            else:
                r, c = p.shape
                lr = 0.04 * 0.7 * max(1.0, math.sqrt(max(r / c, c / r)))
                mom, sec = state.get(n, (torch.zeros_like(p), torch.zeros((r, 1) if r >= c else (1, c), dtype=p.dtype)))
                ref[n], mom, sec = _ref_muon(p, g, mom, sec, 0.9, lr, 0.1, 0.95)
                state[n] = (mom, sec)
                continue
            m, v = state.get(n, (torch.zeros_like(p), torch.zeros_like(p)))
            ref[n], m, v = _ref_adamw(p, g, m, v, t, lr * 0.7, b1, b2, 1e-10)
            state[n] = (m, v)
    for n, p in params.items():
        assert (p.double() - ref[n]).abs().max() < 2e-5, n


def test_schedules():
    assert lr_multiplier(0.2, 0.0, 0.5, 0.0) == 1.0
    assert abs(lr_multiplier(0.75, 0.0, 0.5, 0.0) - 0.5) < 1e-12
    assert abs(lr_multiplier(0.05, 0.1, 0.5, 0.0) - 0.5) < 1e-12
    assert muon_momentum(0) == 0.85 and abs(muon_momentum(150) - 0.90) < 1e-12 and muon_momentum(999) == 0.95
    assert abs(weight_decay_at(0.25, 0.2) - 0.15) < 1e-12


def test_state_roundtrip_and_sharding():
    cfg = GPTConfig(sequence_len=16, vocab_size=64, n_layer=1, n_head=2, n_kv_head=2, n_embd=32)
    model = GPT(cfg)
    owned = {"wte", "layer0_q"}
    opt = MuonAdamW(model.named(), model.param_groups(), model_dim=32, owned=owned)
    assert set(opt.state) == owned
    grads = {n: torch.ones_like(p) for n, p in model.named().items()}
    before = {n: p.detach().clone() for n, p in model.named().items()}
    opt.step(grads)
    for n, p in model.named().items():
        assert torch.equal(p, before[n]) == (n not in owned), n
    t = opt.state_tensors()
    assert set(t) == {"adam_m_wte", "adam_v_wte", "muon_mom_layer0_q", "muon_sec_layer0_q"}
    opt2 = MuonAdamW(model.named(), model.param_groups(), model_dim=32, owned=owned)
    assert opt2.load_state(t, opt.state_steps()) == 4
    assert opt2.state["wte"]["step"] == 1
