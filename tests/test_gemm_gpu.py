"""tcgen05 GEMM vs an fp32 PyTorch matmul of the same bf16 operands, with 256-column tiles run by CTA
pairs (cta_group::2, the default) and by single CTAs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[2, 0], ids=["pair", "single"])
def pair(request, cuda):
    """2: every 256-column GEMM with more than one row tile on CTA pairs (aux epilogues included); 0: none."""
    from bitresearch_b200.ops._ext import ext
    ext().gemm_set_pair(request.param)
    yield request.param
    ext().gemm_set_pair(1)


def _ops():
    from bitresearch_b200.ops import gemm
    from bitresearch_b200.ops._ext import check_status
    return gemm, check_status


def _close(out, ref, K):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= 2e-2 * scale, (err, scale)


def _rand(*shape, dev):
    return (torch.randn(*shape, device=dev) * 0.5).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 512), (300, 520, 200), (1000, 1536, 512), (64, 128, 96)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_majors_and_tails(cuda, pair, M, N, K, a_t, b_t):
    gemm, check_status = _ops()
    torch.manual_seed(0)
    a = _rand(K, M, dev=cuda).t() if a_t else _rand(M, K, dev=cuda)       # logical [M, K]
    b = _rand(N, K, dev=cuda).t() if b_t else _rand(K, N, dev=cuda)       # logical [K, N]
    if (a_t and M % 8) or (b_t and K % 8) or (not b_t and N % 8) or (not a_t and K % 8):
        pytest.skip("TMA row strides must be multiples of 16 bytes")
    out = gemm.matmul(a, b)
    torch.cuda.synchronize()
    assert check_status() == 0
    _close(out, a.float() @ b.float(), K)


def test_gemm_epilogues(cuda, pair):
    gemm, check_status = _ops()
    torch.manual_seed(1)
    M, N, K = 384, 512, 256
    a, b = _rand(M, K, dev=cuda), _rand(K, N, dev=cuda)
    ref = a.float() @ b.float()
    aux = _rand(M, N, dev=cuda)
    _close(gemm.matmul(a, b, epi=gemm.BF16, aux=aux, alpha=0.5, beta=2.0), 0.5 * ref + 2 * aux.float(), K)
    r = torch.randn(M, N, device=cuda)
    out = r.clone()
    gemm.matmul(a, b, out=out, epi=gemm.F32, aux=out, beta=1.0)
    _close(out, ref + r, K)
    _close(gemm.matmul(a, b, epi=gemm.RELU2), torch.relu(ref) ** 2, K)
    h = (torch.relu(torch.randn(M, N, device=cuda)) ** 2).to(torch.bfloat16)
    _close(gemm.matmul(a, b, epi=gemm.RELU2_BWD, aux=h), ref * 2 * h.float().sqrt(), K)
    _close(gemm.matmul(a, b, epi=gemm.SOFTCAP, alpha=1 / 15, beta=15.0), 15 * torch.tanh(ref / 15), K)
    torch.cuda.synchronize()
    assert check_status() == 0


@pytest.mark.parametrize("splits", [1, 4, 0])
def test_gemm_split_k_weight_grad(cuda, pair, splits):
    gemm, check_status = _ops()
    torch.manual_seed(2)
    T, Din, Dout = 8192, 512, 1536
    x, dy = _rand(T, Din, dev=cuda), _rand(T, Dout, dev=cuda)
    acc = torch.randn(Din, Dout, device=cuda)
    ref = acc + x.float().t() @ dy.float()
    gemm.matmul(x.t(), dy, out=acc, epi=gemm.ATOMIC, k_splits=splits)
    torch.cuda.synchronize()
    assert check_status() == 0
    _close(acc, ref, T)


def test_gemm_batched(cuda, pair):
    gemm, check_status = _ops()
    torch.manual_seed(3)
    S, r, c = 6, 512, 256
    X = _rand(S, r, c, dev=cuda)
    A = gemm.matmul(X.mT, X)  # X^T X per matrix (MN-major A and B)
    _close(A, X.float().mT @ X.float(), r)
    Bm = gemm.matmul(A, A, epi=gemm.BF16, aux=A, alpha=0.5, beta=-1.0)
    _close(Bm, 0.5 * (A.float() @ A.float()) - A.float(), c)
    torch.cuda.synchronize()
    assert check_status() == 0


@pytest.mark.parametrize("with_ve", [False, True])
def test_qkv_rope_epilogue_matches_gemm_then_rope(cuda, pair, with_ve):
    """The fused QKV GEMM epilogue (RoPE + QK-norm on q/k heads, VE add on v heads) against the plain
    GEMM followed by the separate RoPE kernel; M = 3 x 100 leaves a partial last row tile."""
    from bitresearch_b200.ops import gemm
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    torch.manual_seed(11)
    T, B, H, KV, D, V = 100, 3, 4, 2, 256, 64
    M, N = B * T, (H + 2 * KV) * 128
    x = torch.randn(M, D, device=cuda).to(torch.bfloat16)
    w = (torch.randn(D, N, device=cuda) * D ** -0.5).to(torch.bfloat16)
    pos = torch.arange(T, device=cuda, dtype=torch.float32)[:, None]
    inv = 10000.0 ** (-torch.arange(0, 128, 2, device=cuda, dtype=torch.float32) / 128)
    cos, sin = torch.cos(pos * inv).contiguous(), torch.sin(pos * inv).contiguous()
    idx = torch.randint(0, V, (M,), device=cuda, dtype=torch.int32)
    ve = torch.randn(V, KV * 128, device=cuda) if with_ve else None
    cur = torch.randn(M, D, device=cuda) if with_ve else None
    wg = torch.randn(32, KV, device=cuda) * 0.3 if with_ve else None
    ref = gemm.matmul(x, w)
    rq0, rk0 = torch.empty(M, H, device=cuda), torch.empty(M, KV, device=cuda)
    gate0 = torch.empty(M, KV, device=cuda) if with_ve else None
    E.rope_fwd(ref, T, H, KV, 128, cos, sin, rq0, rk0, idx, ve, cur, wg, gate0)
    out = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    rq, rk = torch.empty(M, H, device=cuda), torch.empty(M, KV, device=cuda)
    gate = torch.empty(M, KV, device=cuda) if with_ve else None
    gemm.qkv_rope(x, w, out, cos, sin, rq, rk, T, H, KV, idx, ve, cur, wg, gate)
    torch.cuda.synchronize()
    assert check_status() == 0
    # both round the GEMM result to bf16 at different points (before RoPE in the reference path)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(rq, rq0, rtol=1e-2, atol=1e-3)
    torch.testing.assert_close(rk, rk0, rtol=1e-2, atol=1e-3)
    if with_ve:
        torch.testing.assert_close(gate, gate0, rtol=1e-5, atol=1e-5)


def test_pair_and_single_tiles_agree_at_production_shapes(cuda):
    """The same GEMMs with CTA pairs and with single CTAs: forward K = 512 and K = 2048 shapes, an
    MN-major weight-gradient GEMM with split-K, and a row count that leaves the last pair half empty."""
    from bitresearch_b200.ops import gemm
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    torch.manual_seed(5)
    cases = [((16384 + 128, 512), (512, 1536), gemm.BF16), ((8192, 2048), (2048, 512), gemm.BF16),
             ((8192, 512), (512, 2048), gemm.RELU2)]
    try:
        for (m, k), (k2, n), epi in cases:
            a, b = _rand(m, k, dev=cuda), _rand(k2, n, dev=cuda)
            E.gemm_set_pair(2)
            p = gemm.matmul(a, b, epi=epi)
            E.gemm_set_pair(0)
            s1 = gemm.matmul(a, b, epi=epi)
            torch.cuda.synchronize()
            assert check_status() == 0
            torch.testing.assert_close(p.float(), s1.float(), rtol=1e-2, atol=1e-2)
        x, dy = _rand(8192, 512, dev=cuda), _rand(8192, 2048, dev=cuda)
        outs = []
        for on in (2, 0):
            E.gemm_set_pair(on)
            o = torch.zeros(512, 2048, device=cuda)
            gemm.matmul(x.t(), dy, out=o, epi=gemm.ATOMIC, k_splits=0)
            outs.append(o)
        torch.cuda.synchronize()
        assert check_status() == 0
        _close(outs[0], x.float().t() @ dy.float(), 8192)
        torch.testing.assert_close(outs[0], outs[1], rtol=1e-3, atol=1e-2)
    finally:
        E.gemm_set_pair(1)
