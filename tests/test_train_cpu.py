"""Trainer on CPU: loss decreases, gloo DP ranks stay in lock-step, checkpoint resume is exact."""
import numpy as np
import torch

from dist_utils import run_world
from bitresearch_b200.config import apply_overrides, preset
from bitresearch_b200.train import Trainer


def _cfg(**kw):
    c = preset("tiny-cpu")
    c = apply_overrides(c, ["model.n_layer=2", "model.n_embd=64", "model.n_head=2", "model.n_kv_head=2",
                            "model.sequence_len=32", "model.vocab_size=128", "device_batch=4",
                            "total_batch_tokens=128", "eval_tokens=256", "log_every=0", "results_tsv="])
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def test_loss_decreases_and_summary(capsys):
    cfg = _cfg(max_steps=25, time_budget=1e9, data="zipf", doc_mean_len=32)
    tr = Trainer(cfg, device="cpu")
    tr.initialize()
    first = tr.train_step()
    m = tr.start_training()
    assert m.step == 25 and m.loss < first - 0.3
    out = capsys.readouterr().out
    assert "\nval_bpb:" in out and "num_params_M:" in out and m.val_bpb > 0


def test_markov_data_reports_its_loss_floor(capsys):
    cfg = _cfg(max_steps=30, time_budget=1e9, data="markov", doc_mean_len=32)
    tr = Trainer(cfg, device="cpu")
    tr.initialize()
    m = tr.start_training()
    out = capsys.readouterr().out
    floor = float(out.split("val_bpb_floor:")[1].split()[0])
    assert 0 < floor < m.val_bpb
    assert m.extra["val_nats_floor"] < m.loss


def _dp(rank, world, comm, sparsify):
    cfg = _cfg(max_steps=4, comm=comm, total_batch_tokens=128 * world)
    cfg.sparsify.enabled = sparsify
    cfg.sparsify.warmup_steps = 2
    tr = Trainer(cfg, device="cpu", log=lambda m: None)
    tr.initialize()
    for _ in range(4):
        tr.train_step()
    return {n: p.detach().numpy().copy() for n, p in tr.model.named().items()}


def test_gloo_dp_ring_ranks_identical():
    r0, r1 = run_world(_dp, 2, "ring", False)
    for n in r0:
        assert np.array_equal(r0[n], r1[n]), n


def test_gloo_dp_process_group_all_reduce_ranks_identical():
    # comm=nccl: one all-reduce of the flat gradient over the default group (gloo here), replicated optimizer
    r0, r1 = run_world(_dp, 2, "nccl", False)
    for n in r0:
        assert np.array_equal(r0[n], r1[n]), n


def test_gloo_dp_topk_sparsified_ring():
    r0, r1 = run_world(_dp, 2, "ring", True)
    for n in r0:
        assert np.array_equal(r0[n], r1[n]), n


def _time_budget(rank, world):
    import time
    cfg = _cfg(max_steps=10_000, comm="ring", total_batch_tokens=128 * world, time_budget=1.5,
               warmup_steps_excluded=2)
    tr = Trainer(cfg, device="cpu", log=lambda m: None)
    tr.initialize()
    step = tr.train_step
    if rank == 1:  # the slower rank: its clock alone would keep it training after rank 0 stops

        def slow(*a, **k):
            time.sleep(0.02)
            return step(*a, **k)

        tr.train_step = slow
    m = tr.start_training()
    p = np.concatenate([v.detach().numpy().ravel() for v in tr.model.named().values()])
    return m.step, tr.total_training_time, p


def test_gloo_time_budget_stops_every_rank_on_the_same_step():
    (s0, t0, p0), (s1, t1, p1) = run_world(_time_budget, 2, timeout=120)
    assert s0 == s1 and s0 > 3
    assert t0 == t1 >= 1.5
    assert np.array_equal(p0, p1)


def test_checkpoint_resume_reproduces_trajectory(tmp_path):
    cfg = _cfg(max_steps=10)
    a = Trainer(cfg, device="cpu", log=lambda m: None)
    a.initialize()
    for _ in range(3):
        a.train_step()
    path = a.save_checkpoint(str(tmp_path / "c.safetensors"))
    la = [a.train_step() for _ in range(3)]
    b = Trainer(cfg, device="cpu", log=lambda m: None)
    b.initialize()
    b.load_checkpoint(path)
    # the data stream is positioned by step count: replay the consumed batches
    for _ in range(3):
        b.next_batch()
    lb = [b.train_step() for _ in range(3)]
    assert b.metrics.step == 6
    np.testing.assert_allclose(la, lb, rtol=0, atol=0)
    for n, p in a.model.named().items():
        assert torch.equal(p, b.model.named()[n]), n


def test_cli_peers_launches_ranks(tmp_path):
    import os
    import subprocess
    import sys
    out = subprocess.run([sys.executable, "-m", "bitresearch_b200.train", "--preset", "tiny-cpu", "--peers", "2",
                          "--max-steps", "2", "comm=ring", "eval_tokens=512", "results_tsv=", "log_every=1",
                          "model.n_layer=1"], capture_output=True, text=True, timeout=240,
                         cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert out.returncode == 0, out.stderr[-2000:]
    assert "world=2" in out.stdout and "num_steps:        2" in out.stdout and "peers=2" in out.stdout


def test_profiler_hook_writes_a_chrome_trace(tmp_path):
    import json
    cfg = _cfg(max_steps=4, time_budget=1e9, profile_steps="1:3", profile_dir=str(tmp_path))
    tr = Trainer(cfg, device="cpu", log=lambda m: None)
    tr.initialize()
    tr.start_training()
    path = tmp_path / "trace_rank0_steps1-3.json"
    assert path.exists()
    ev = json.loads(path.read_text())
    assert len(ev["traceEvents"]) > 10


def test_same_seed_replays_bitwise_on_cpu():
    def run():
        tr = Trainer(_cfg(max_steps=5), device="cpu", log=lambda m: None)
        tr.initialize()
        return [float(tr.train_step()) for _ in range(5)]

    assert run() == run()
