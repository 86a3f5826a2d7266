"""Index checks of the kernels that gather or scatter table rows by token id or target: an id outside the
table records kErrBadIndex (6) in the device status word and that row's table access is skipped; every
other row is computed as usual. The tables are views into larger buffers, so the rows just past them
are allocated memory of this test."""
import pytest
import torch

pytestmark = pytest.mark.gpu

BAD_INDEX = 6


def _rms(x):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5)


def test_embedding_skips_and_reports_an_id_outside_the_table(cuda):
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    check_status()
    V, M, D = 100, 64, 512
    big = torch.randn(V + 8, D, device=cuda)
    wte = big[:V]
    idx = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    idx[9] = V
    x0 = torch.full((M, D), 3.0, device=cuda)
    r0 = torch.empty(M, device=cuda)
    E.embed_rms_fwd(idx, wte, x0, r0)
    torch.cuda.synchronize()
    assert check_status() == BAD_INDEX
    ok = torch.ones(M, dtype=torch.bool, device=cuda)
    ok[9] = False
    torch.testing.assert_close(x0[ok], _rms(wte[idx[ok].long()]), rtol=1e-5, atol=1e-5)
    assert x0[9].abs().max().item() == 0.0 and r0[9].item() == 0.0
    dbig = torch.zeros(V + 8, D, device=cuda)
    E.embed_bwd(idx, wte, r0, torch.randn(M, D, device=cuda), dbig[:V])
    torch.cuda.synchronize()
    assert check_status() == BAD_INDEX
    assert dbig[V:].abs().max().item() == 0.0  # nothing written past the table


def test_cross_entropy_masks_and_reports_a_target_outside_the_vocabulary(cuda):
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    check_status()
    M, D, V = 256, 512, 1000
    x = (torch.randn(M, D, device=cuda)).to(torch.bfloat16)
    wbig = torch.randn(V + 8, D, device=cuda) * 0.05
    w = wbig[:V]
    tgt = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    tgt[5] = V + 3
    tgt[6] = -1
    G = torch.empty(M, V, dtype=torch.bfloat16, device=cuda)
    part = torch.empty(2 * ((V + 255) // 256), M, device=cuda)
    zt = torch.empty(M, device=cuda)
    rs, cf = torch.empty(M, device=cuda), torch.empty(M, device=cuda)
    nats = torch.empty(M, device=cuda)
    loss = torch.zeros(1, device=cuda)
    dwbig = torch.zeros(V + 8, D, device=cuda)
    xs = torch.empty_like(x)
    E.gemm_softcap_ce(x, w.to(torch.bfloat16), G, tgt, part, zt, 15.0, True)
    E.ce_finalize(part, zt, tgt, V, 15.0, 1.0 / M, nats=nats, loss_sum=loss, rowscale=rs, coef=cf, x=x, xs=xs,
                  dw=dwbig[:V])
    torch.cuda.synchronize()
    assert check_status() == BAD_INDEX
    assert nats[5].item() == 0.0 and rs[5].item() == 0.0 and cf[5].item() == 0.0
    assert nats[6].item() == 0.0 and rs[6].item() == 0.0
    assert (nats[7:] > 0).all() and torch.isfinite(loss).all()
    assert dwbig[V:].abs().max().item() == 0.0
    # -1 alone is the ignore value, not an error
    tgt[5] = 1
    E.ce_finalize(part, zt, tgt, V, 15.0, 1.0 / M, nats=nats)
    torch.cuda.synchronize()
    assert check_status() == 0
