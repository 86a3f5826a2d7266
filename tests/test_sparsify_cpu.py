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


def _residual_after(masking, steps=12):
    sp = GradientSparsifier(top_k_ratio=0.01, warmup_steps=0, sample_size=1000, momentum_factor=0.9, seed=0,
                            momentum_masking=masking)
    n = 1000
    for _ in range(steps):
        g = torch.full((n,), 1e-3)
        g[:20] = 1.0  # these fill the top 1% every step, the constant small gradient is never sent
        sp.sparsify(g)
    return float(sp.error[20:].abs().max())


def test_reference_momentum_residual_grows_geometrically_masked_one_linearly():
    # reference update: e <- (1 + mu) e + g for an unsent entry; DGC: v grows by u -> g / (1 - mu) per step
    ref = _residual_after(False)
    dgc = _residual_after(True)
    assert ref > 1e-3 * 1.9 ** 11
    assert dgc < 1e-3 * 12 / (1 - 0.9)


def test_momentum_masking_clears_sent_velocity():
    sp = GradientSparsifier(top_k_ratio=0.1, warmup_steps=0, sample_size=100, momentum_factor=0.5, seed=0,
                            momentum_masking=True)
    g = torch.full((100,), 0.01)
    g[:20] = 1.0  # 20% large entries hold the 10% threshold at 1.0
    for step in range(2):
        s = sp.sparsify(g.clone())
        assert sorted(s.indices.tolist()) == list(range(20))
        assert (sp.velocity[:20] == 0).all() and (sp.error[:20] == 0).all()
    # unsent: u1 = 0.01, v1 = 0.01; u2 = 0.5 u1 + 0.01 = 0.015, v2 = v1 + u2 = 0.025
    assert torch.allclose(sp.velocity[20:], torch.full((80,), 0.015))
    assert torch.allclose(sp.error[20:], torch.full((80,), 0.025))
