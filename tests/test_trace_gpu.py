"""Phase tracing and replay on one B200: CUDA-event phases per step, and two runs from the same seed.

The fused engine accumulates some reductions with fp32 atomics (split-K weight gradients, embedding
scatter-add), whose order varies from run to run; the first step's loss (before any update) must
match to rounding, later steps to a small tolerance."""
import pytest

pytestmark = pytest.mark.gpu


def _trainer(**kw):
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.train import Trainer
    cfg = apply_overrides(preset("d512"), ["model.n_layer=2", "device_batch=8", "total_batch_tokens=32768",
                                           "log_every=0", "results_tsv=", "eval_tokens=32768"])
    for k, v in kw.items():
        setattr(cfg, k, v)
    tr = Trainer(cfg, log=lambda m: None)
    tr.initialize()
    return tr


def test_phase_timer_reports_every_phase(cuda):
    tr = _trainer(trace_phases=True)
    for _ in range(2):
        tr.train_step()
    ph = tr.phase_ms
    assert {"data", "forward", "backward", "sync_update"} <= set(ph), ph
    assert all(v > 0 for v in ph.values())
    assert ph["backward"] > ph["forward"] * 0.8  # backward does about twice the forward's work
    tr.destroy()


def test_same_seed_replays_on_gpu(cuda):
    def run():
        tr = _trainer(data="markov")
        out = [float(tr.train_step()) for _ in range(5)]
        tr.destroy()
        return out

    a, b = run(), run()
    assert abs(a[0] - b[0]) <= 1e-6 * abs(a[0])
    assert all(abs(x - y) <= 2e-3 * abs(x) for x, y in zip(a, b)), (a, b)
