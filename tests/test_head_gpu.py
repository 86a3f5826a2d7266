"""The fused lm_head + softcap + cross-entropy (gemm_softcap_ce -> ce_finalize -> dW GEMM and rms_bwd's head
form) against an fp32 PyTorch reference of the final RMSNorm, the lm_head, the softcap and the reference's
cross-entropy (``-log(softmax + 1e-10)``, masked mean over all positions; src/model/gpt.ts:296-313)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

CAP = 15.0


def _assert(a, b, tol, what):
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item() + 1e-12
    assert err <= tol * scale, (what, err, scale)


@pytest.fixture(params=[1, 0], ids=["pairs", "single"])
def pair(request, cuda):
    """1: the default CTA-pair policy (the head GEMM on pairs with eight epilogue warps); 0: single CTAs
    with four."""
    from bitresearch_b200.ops._ext import ext
    ext().gemm_set_pair(request.param)
    yield request.param
    ext().gemm_set_pair(1)


@pytest.mark.parametrize("form", ["patch", "scatter"])
@pytest.mark.parametrize("V", [1000, 8192, 65536])
def test_fused_head_matches_fp32_reference(cuda, V, form, pair):
    """form "patch" (the engine's): ce_finalize writes the target column's gradient into G; "scatter": it
    scatters it into dW in fp32 and rms_bwd adds it to dx."""
    from bitresearch_b200.ops import gemm
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    torch.manual_seed(V)
    M, D = 300, 512
    h = torch.randn(M, D, device=cuda)                        # final residual stream (fp32)
    w = torch.randn(V, D, device=cuda) * 0.05                 # lm_head table (fp32 master)
    wb = w.to(torch.bfloat16)
    tgt = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    tgt[[3, 77, 299]] = -1                                     # ignored positions
    scale = 1.0 / M

    # kernel path
    xf = torch.empty(M, D, dtype=torch.bfloat16, device=cuda)
    rstd = torch.empty(M, device=cuda)
    E.rms_fwd(h, xf, rstd)
    nt = (V + 255) // 256
    G = torch.empty(M, V, dtype=torch.bfloat16, device=cuda)
    part = torch.empty(2 * nt, M, device=cuda)
    zt = torch.empty(M, device=cuda)
    rs = torch.empty(M, device=cuda)
    cf = torch.empty(M, device=cuda)
    xs = torch.empty(M, D, dtype=torch.bfloat16, device=cuda)
    nats = torch.empty(M, device=cuda)
    loss = torch.zeros(1, device=cuda)
    dw = torch.zeros(V, D, device=cuda)
    E.gemm_softcap_ce(xf, wb, G, tgt, part, zt, CAP, True)
    if form == "patch":
        E.ce_finalize(part, zt, tgt, V, CAP, scale, nats=nats, loss_sum=loss, rowscale=rs, x=xf, xs=xs, g=G)
    else:
        E.ce_finalize(part, zt, tgt, V, CAP, scale, nats=nats, loss_sum=loss, rowscale=rs, coef=cf, x=xf, xs=xs,
                      dw=dw)
    gemm.matmul(G.t(), xs, out=dw, epi=gemm.ATOMIC, k_splits=0)
    raw = torch.empty(M, D, device=cuda)
    gemm.matmul(G, wb, out=raw, epi=gemm.F32)
    dh = torch.empty(M, D, device=cuda)
    if form == "patch":
        E.rms_bwd(h, rstd, raw, None, dh, None, rs)
    else:
        E.rms_bwd(h, rstd, raw, None, dh, None, rs, cf, tgt, w)
    # evaluation form: statistics only, no G written
    nats_eval = torch.empty(M, device=cuda)
    G2 = torch.full((M, V), 7.0, dtype=torch.bfloat16, device=cuda)
    E.gemm_softcap_ce(xf, wb, G2, tgt, part, zt, CAP, False)
    E.ce_finalize(part, zt, tgt, V, CAP, 1.0, nats=nats_eval)
    torch.cuda.synchronize()
    assert check_status() == 0

    # fp32 reference on the same bf16-rounded GEMM inputs (straight-through for the rounding of rms(h))
    hr = h.clone().requires_grad_()
    wr = wb.float().requires_grad_()
    xn = hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + 1e-5)
    xn_b = xn + (xf.float() - xn).detach()
    logits = CAP * torch.tanh((xn_b @ wr.t()) / CAP)
    p = torch.softmax(logits, -1)
    valid = tgt >= 0
    pt = p.gather(1, tgt.long().clamp(min=0)[:, None]).squeeze(1)
    nll = -torch.log(pt + 1e-10)
    ref_loss = (nll * valid).sum() * scale
    ref_loss.backward()

    assert abs(loss.item() - ref_loss.item()) <= 2e-4 * ref_loss.item(), (loss.item(), ref_loss.item())
    ref_nats = torch.where(valid, nll, torch.zeros_like(nll)).detach()
    assert (nats - ref_nats).abs().max().item() < 2e-3
    assert (nats_eval - ref_nats).abs().max().item() < 2e-3
    assert torch.all(G2 == 7.0), "the evaluation form wrote G"
    _assert(dw, wr.grad, 2e-2, "dW")
    _assert(dh, hr.grad, 2e-2, "dh")
    # the rows of ignored positions get no gradient
    assert dh[[3, 77, 299]].abs().max().item() == 0.0
