import torch

from bitresearch_b200.parallel.sparsify import GradientSparsifier


def test_error_feedback_invariant_and_kept_fraction():
    sp = GradientSparsifier(top_k_ratio=0.1, warmup_steps=2, sample_size=5000, momentum_factor=0.0, seed=0)
    g0 = torch.randn(20000)
    d = sp.sparsify(g0.clone())  # dense warm-up (the reference counts the step before checking, so warmup_steps=2 gives one dense step)
    assert d.indices.numel() == 20000
    prev_err = torch.zeros(20000)
    for _ in range(3):
        g = torch.randn(20000)
        inp = g.clone()
        s = sp.sparsify(g)
        sent = GradientSparsifier.densify(s)
        torch.testing.assert_close(sent + sp.error, inp + prev_err)  # nothing is lost
        assert torch.equal(g, sent)  # the dense buffer is zeroed outside the kept set
        frac = s.indices.numel() / 20000
        assert 0.07 < frac < 0.13
        prev_err = sp.error.clone()


def test_momentum_correction_and_codec():
    sp = GradientSparsifier(top_k_ratio=0.25, warmup_steps=0, sample_size=100, momentum_factor=0.9, seed=1)
    g = torch.randn(1000)
    s = sp.sparsify(g.clone())
    assert torch.allclose(sp.velocity, g)
    buf = GradientSparsifier.encode(s)
    assert len(buf) == 8 + 8 * s.indices.numel()
    r = GradientSparsifier.decode(buf)
    assert r.length == 1000 and torch.equal(r.indices, s.indices) and torch.equal(r.values, s.values)
    assert abs(GradientSparsifier.compression_ratio(s) - len(buf) / 4000) < 1e-12
