"""Row kernels, RoPE/QK-norm/VE, fused cross-entropy, attention and optimizer kernels vs fp32 PyTorch."""
import math

import numpy as np

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ext():
    from bitresearch_b200.ops._ext import ext
    return ext()


def _rms(x):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5)


def _assert(a, b, tol):
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item() + 1e-6
    assert err <= tol * scale, (err, scale)


def test_embed_ladder_rms_fwd_bwd(cuda):
    E = _ext()
    torch.manual_seed(0)
    V, M, D = 300, 777, 512
    idx = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    wte = torch.randn(V, D, device=cuda)
    x0 = torch.empty(M, D, device=cuda)
    r0 = torch.empty(M, device=cuda)
    E.embed_rms_fwd(idx, wte, x0, r0)
    _assert(x0, _rms(wte[idx.long()]), 1e-5)
    x = torch.randn(M, D, device=cuda)
    lam_r = torch.tensor([1.3, 0.7], device=cuda)
    lam_0 = torch.tensor([0.1, 0.4], device=cuda)
    cur = torch.empty(M, D, device=cuda)
    xn = torch.empty(M, D, device=cuda, dtype=torch.bfloat16)
    rs = torch.empty(M, device=cuda)
    E.ladder_rms_fwd(x, x0, lam_r, lam_0, 1, cur, xn, rs)
    ref_cur = 0.7 * x + 0.4 * x0
    _assert(cur, ref_cur, 1e-6)
    _assert(xn, _rms(ref_cur), 1e-2)
    # ladder backward against autograd
    xa, x0a = x.clone().requires_grad_(), x0.clone().requires_grad_()
    la, l0 = lam_r.clone().requires_grad_(), lam_0.clone().requires_grad_()
    c = la[1] * xa + l0[1] * x0a
    y = _rms(c)
    gy = torch.randn_like(y).to(torch.bfloat16)
    dres = torch.randn_like(y)
    dgin = torch.randn(M, 32, device=cuda)
    loss = (y * gy.float()).sum() + (c * dres).sum() + (c[:, :32] * dgin).sum()
    loss.backward()
    dx = torch.empty(M, D, device=cuda)
    dx0 = torch.zeros(M, D, device=cuda)
    dlr = torch.zeros(2, device=cuda)
    dl0 = torch.zeros(2, device=cuda)
    E.ladder_bwd(x, x0, lam_r, lam_0, 1, rs, gy, dres, dgin, dx, dx0, dlr, dl0, False)
    _assert(dx, xa.grad, 1e-4)
    _assert(dx0, x0a.grad, 1e-4)
    assert abs(dlr[1].item() - la.grad[1].item()) < 1e-3 * abs(la.grad[1].item()) + 1e-2
    assert abs(dl0[1].item() - l0.grad[1].item()) < 1e-3 * abs(l0.grad[1].item()) + 1e-2
    # rms backward with residual
    xr = torch.randn(M, D, device=cuda, requires_grad=True)
    gy2 = torch.randn(M, D, device=cuda)
    (_rms(xr) * gy2).sum().backward()
    rr = torch.rsqrt(xr.detach().pow(2).mean(-1) + 1e-5)
    out = torch.empty(M, D, device=cuda)
    outb = torch.empty(M, D, device=cuda, dtype=torch.bfloat16)
    E.rms_bwd(xr.detach(), rr, gy2, dres, out, outb)
    _assert(out, xr.grad + dres, 1e-4)
    _assert(outb, xr.grad + dres, 1e-2)
    # embedding scatter backward
    wa = wte.clone().requires_grad_()
    ga = torch.randn(M, D, device=cuda)
    (_rms(wa[idx.long()]) * ga).sum().backward()
    dw = torch.zeros_like(wte)
    E.embed_bwd(idx, wte, r0, ga, dw)
    _assert(dw, wa.grad, 1e-4)


def _rope_ref(qkv, T, H, KV, hd, cos, sin, idx, ve, cur, wg):
    M = qkv.shape[0]
    q = qkv[:, :H * hd].view(M, H, hd)
    k = qkv[:, H * hd:(H + KV) * hd].view(M, KV, hd)
    v = qkv[:, (H + KV) * hd:].view(M, KV, hd)
    t = torch.arange(M, device=qkv.device) % T
    c, s = cos[t].view(M, 1, hd // 2), sin[t].view(M, 1, hd // 2)

    def rot(x):
        x1, x2 = x[..., :hd // 2], x[..., hd // 2:]
        return torch.cat([x1 * c + x2 * s, -x1 * s + x2 * c], -1)
    q = _rms(rot(q))
    k = _rms(rot(k))
    gate = 2 * torch.sigmoid(cur[:, :32] @ wg)
    v = v + ve[idx.long()].view(M, KV, hd) * gate.view(M, KV, 1)
    return torch.cat([q.reshape(M, -1), k.reshape(M, -1), v.reshape(M, -1)], 1), gate


@pytest.mark.parametrize("hd", [128, 64])
def test_rope_qknorm_ve(cuda, hd):
    E = _ext()
    torch.manual_seed(1)
    B, T, H, KV, V = 2, 64, 4, 2, 50
    M = B * T
    D = H * hd
    qkv = torch.randn(M, (H + 2 * KV) * hd, device=cuda)
    inv = 1.0 / (10000 ** (torch.arange(0, hd, 2, device=cuda).float() / hd))
    fr = torch.outer(torch.arange(T, device=cuda).float(), inv)
    cos, sin = fr.cos().contiguous(), fr.sin().contiguous()
    idx = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    ve = torch.randn(V, KV * hd, device=cuda) * 0.1
    cur = torch.randn(M, D, device=cuda)
    wg = torch.randn(32, KV, device=cuda) * 0.1
    qkv_b = qkv.to(torch.bfloat16)
    ref_in = qkv_b.float().requires_grad_()
    ve_a = ve.clone().requires_grad_()
    cur_a = cur.clone().requires_grad_()
    wg_a = wg.clone().requires_grad_()
    ref, gate_ref = _rope_ref(ref_in, T, H, KV, hd, cos, sin, idx, ve_a, cur_a, wg_a)
    buf = qkv_b.clone()
    rq = torch.empty(M, H, device=cuda)
    rk = torch.empty(M, KV, device=cuda)
    gate = torch.empty(M, KV, device=cuda)
    E.rope_fwd(buf, T, H, KV, hd, cos, sin, rq, rk, idx, ve, cur, wg, gate)
    _assert(buf, ref, 2e-2)
    _assert(gate, gate_ref, 1e-4)
    g = torch.randn_like(ref).to(torch.bfloat16)
    (ref * g.float()).sum().backward()
    dq = g.clone()
    dve = torch.zeros_like(ve)
    dz = torch.empty(M, KV, device=cuda)
    E.rope_bwd(dq, buf, T, H, KV, hd, cos, sin, rq, rk, idx, ve, gate, dve, dz)
    _assert(dq, ref_in.grad, 3e-2)
    _assert(dve, ve_a.grad, 2e-2)
    dwg = torch.zeros_like(wg)
    dgin = torch.empty(M, 32, device=cuda)
    E.ve_gate_bwd(cur, dz, wg, dwg, dgin)
    _assert(dwg, wg_a.grad, 2e-2)
    _assert(dgin, cur_a.grad[:, :32], 2e-2)


@pytest.mark.parametrize("V", [8192, 1000])
def test_softcap_ce(cuda, V):
    E = _ext()
    torch.manual_seed(2)
    M = 300
    z = (torch.randn(M, V, device=cuda) * 8).requires_grad_()
    tgt = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    tgt[5] = -1
    logits = 15 * torch.tanh(z / 15)
    lb = logits.detach().to(torch.bfloat16)
    lf = lb.float()
    p = torch.softmax(lf, -1)
    nll = -torch.log(p.gather(1, tgt.long().clamp(min=0)[:, None]).squeeze(1) + 1e-10)
    valid = (tgt != -1).float()
    loss = (nll * valid).sum() / M
    # gradient of the reference loss w.r.t. z through the bf16 logits
    lf2 = lf.clone().requires_grad_()
    p2 = torch.softmax(lf2, -1)
    l2 = ((-torch.log(p2.gather(1, tgt.long().clamp(min=0)[:, None]).squeeze(1) + 1e-10)) * valid).sum() / M
    l2.backward()
    dz_ref = lf2.grad * (1 - (lf / 15) ** 2)
    buf = lb.clone()
    nats = torch.empty(M, device=cuda)
    ls = torch.zeros(1, device=cuda)
    E.softcap_ce(buf, tgt, 15.0, 1.0 / M, nats, ls, True)
    assert abs(ls.item() - loss.item()) < 1e-4 * loss.item()
    _assert(nats, nll, 1e-4)
    _assert(buf, dz_ref, 2e-2)


def _attn_ref(q, k, v, window):
    B, T, H, hd = q.shape
    KV = k.shape[2]
    k = k.repeat_interleave(H // KV, 2)
    v = v.repeat_interleave(H // KV, 2)
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(hd)
    i = torch.arange(T, device=q.device)[:, None]
    j = torch.arange(T, device=q.device)[None]
    mask = (j <= i) & (j > i - window)
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, -1)
    return torch.einsum("bhqk,bkhd->bqhd", p, v), torch.logsumexp(s, -1)


@pytest.mark.parametrize("B,T,H,KV,window,hd", [(2, 256, 4, 4, 256, 128), (1, 300, 4, 2, 100, 128),
                                                (2, 512, 2, 2, 128, 128), (1, 193, 2, 1, 1000, 128),
                                                (2, 1024, 2, 1, 300, 128), (1, 2048, 2, 2, 1024, 128),
                                                (1, 640, 4, 2, 200, 128), (2, 384, 2, 2, 384, 128),
                                                (2, 512, 4, 4, 256, 64), (1, 300, 4, 2, 100, 64),
                                                (1, 193, 2, 1, 1000, 64)])
def test_attention_fwd_bwd(cuda, B, T, H, KV, window, hd):
    E = _ext()
    torch.manual_seed(3)
    tc = T % 128 == 0 and hd == 128  # the tcgen05 kernels: 128-wide heads, whole 128-row tiles
    D, Dkv = H * hd, KV * hd
    M = B * T
    qkv = (torch.randn(M, D + 2 * Dkv, device=cuda)).to(torch.bfloat16)
    q, k, v = qkv[:, :D], qkv[:, D:D + Dkv], qkv[:, D + Dkv:]
    o = torch.empty(M, D, device=cuda, dtype=torch.bfloat16)
    lse = torch.empty(B, H, T, device=cuda)
    E.attn_fwd(q, k, v, o, lse, B, T, H, KV, hd, window)
    if tc:
        o_tc = torch.empty_like(o)
        lse_tc = torch.empty_like(lse)
        E.attn_fwd_tc(qkv, o_tc, lse_tc, B, T, H, KV, hd, window)
        torch.cuda.synchronize()
        from bitresearch_b200.ops._ext import check_status
        assert check_status() == 0
    qr = q.float().view(B, T, H, hd).requires_grad_()
    kr = k.float().view(B, T, KV, hd).requires_grad_()
    vr = v.float().view(B, T, KV, hd).requires_grad_()
    ref, lse_ref = _attn_ref(qr, kr, vr, min(window, T))
    _assert(o, ref.reshape(M, D), 2e-2)
    _assert(lse, lse_ref, 1e-3)
    if tc:
        _assert(o_tc, ref.reshape(M, D), 2e-2)
        _assert(lse_tc * math.log(2.0), lse_ref, 1e-3)  # the tcgen05 kernel reports lse in log2 units
    do = torch.randn(M, D, device=cuda).to(torch.bfloat16)
    (ref.reshape(M, D) * do.float()).sum().backward()
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(B, H, T, device=cuda)
    E.attn_bwd(q, k, v, o, do, lse, dqkv[:, :D], dqkv[:, D:D + Dkv], dqkv[:, D + Dkv:], delta, delta, B, T, H, KV,
               hd, window)
    _assert(dqkv[:, :D], qr.grad.reshape(M, D), 3e-2)
    _assert(dqkv[:, D:D + Dkv], kr.grad.reshape(M, Dkv), 3e-2)
    _assert(dqkv[:, D + Dkv:], vr.grad.reshape(M, Dkv), 3e-2)
    if tc:
        dqkv_tc = torch.empty_like(qkv)
        delta_tc = torch.empty(B, H, T, device=cuda)
        E.attn_bwd_tc(qkv, o_tc, do, lse_tc, dqkv_tc, delta_tc, B, T, H, KV, hd, window)
        torch.cuda.synchronize()
        from bitresearch_b200.ops._ext import check_status
        assert check_status() == 0
        _assert(dqkv_tc[:, :D], qr.grad.reshape(M, D), 3e-2)
        _assert(dqkv_tc[:, D:D + Dkv], kr.grad.reshape(M, Dkv), 3e-2)
        _assert(dqkv_tc[:, D + Dkv:], vr.grad.reshape(M, Dkv), 3e-2)


def test_adamw_and_muon_kernels_match_torch_optimizer(cuda):
    """The fused step (bf16 Newton-Schulz on tcgen05) must be as close to an fp32 Newton-Schulz step as
    the eager bf16 step is; AdamW parameters must match the eager step to fp32 rounding."""
    from bitresearch_b200.config import GPTConfig
    from bitresearch_b200.models.gpt import GPT
    from bitresearch_b200.optim.muon_adamw import MuonAdamW
    torch.manual_seed(4)
    cfg = GPTConfig(sequence_len=64, vocab_size=512, n_layer=2, n_head=2, n_kv_head=2, n_embd=256)
    models = [GPT(cfg, device=cuda) for _ in range(3)]
    for m in models[1:]:
        m.load_state_dict(models[0].state_dict())
    ref32 = MuonAdamW(models[0].named(), models[0].param_groups(), model_dim=256, ns_dtype="fp32", impl="torch")
    eager = MuonAdamW(models[1].named(), models[1].param_groups(), model_dim=256, ns_dtype="bf16", impl="torch")
    shadows = {n: torch.empty_like(p, dtype=torch.bfloat16) for n, p in models[2].named().items() if p.dim() == 2}
    fused = MuonAdamW(models[2].named(), models[2].param_groups(), model_dim=256, ns_dtype="bf16", impl="cuda",
                      shadows=shadows)
    init = {n: p.detach().clone() for n, p in models[0].named().items()}
    for o in (ref32, eager, fused):
        o.lr_multiplier, o.muon_momentum, o.muon_weight_decay = 0.9, 0.9, 0.1
    for _ in range(3):
        grads = {n: torch.randn_like(p) * 0.01 for n, p in models[0].named().items()}
        for o in (ref32, eager, fused):
            o.step(grads)
    for n, p32 in models[0].named().items():
        pe, pf = models[1].named()[n], models[2].named()[n]
        moved = (p32 - init[n]).abs().max().item() + 1e-8
        err_eager = (pe - p32).abs().max().item()
        err_fused = (pf - p32).abs().max().item()
        if p32.dim() == 2 and n.startswith("layer") and not n.endswith("ve_gate"):
            assert err_fused <= 1.5 * err_eager + 0.02 * moved, (n, err_fused, err_eager, moved)
        else:
            assert err_fused <= 1e-4 * moved + 1e-6, (n, err_fused, moved)
    for n, s in shadows.items():
        _assert(s, models[2].named()[n], 1e-2)


def test_monte_carlo_sharpe_kernel_distribution(cuda):
    """The GPU Monte-Carlo Sharpe kernel against the numpy restatement: different random streams, so
    the distribution statistics are compared (200k paths: standard errors about 0.002)."""
    from bitresearch_b200.swarm.strategy import mc_sharpes, mc_sharpes_numpy
    for mu, sigma in ((0.0, 0.2), (0.15, 0.1)):
        g = mc_sharpes(mu, sigma, 200_000, seed=7, device=cuda)
        c = mc_sharpes_numpy(mu, sigma, 200_000, seed=7)
        assert abs(g.mean() - c.mean()) < 0.02, (mu, sigma, g.mean(), c.mean())
        assert abs(g.std() - c.std()) < 0.02
        assert abs(np.percentile(g, 5) - np.percentile(c, 5)) < 0.03
        assert abs(np.percentile(g, 95) - np.percentile(c, 95)) < 0.03
