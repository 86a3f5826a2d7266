"""Failure detection and elastic recovery on CPU gloo ranks (no GPU involved): a rank that crashes
between steps stops its heartbeat; the survivors' next collective fails, the step's update is skipped,
they wait until membership drops the lost peer, form a smaller ring with a new gloo group, re-sync the
state from the new position 0 and finish the run with identical weights. A process that joins the room
later (a restarted rank) is taken into the ring, receives the state and finishes in lock-step too."""
import time

import numpy as np

from dist_utils import run_world
from bitresearch_b200.config import apply_overrides, preset
from bitresearch_b200.train import Trainer


class _Crash(Exception):
    pass


def _cfg(world, extra):
    return apply_overrides(preset("tiny-cpu"), [
        "model.n_layer=1", "model.n_embd=64", "model.n_head=1", "model.n_kv_head=1", "model.sequence_len=32",
        "model.vocab_size=128", "device_batch=2", f"total_batch_tokens={64 * world}", "eval_tokens=128",
        "log_every=0", "results_tsv=", "max_steps=8", "time_budget=1e9", "comm=ring", "elastic=true",
        "heartbeat_s=0.2", "dead_after_s=3", "comm_timeout_s=4", "reform_timeout_s=60", *extra])


def _elastic(rank, world, crash_rank, crash_after, extra=(), rejoin=False, join_delay_s=0.0):
    cfg = _cfg(world, extra)
    logs = []
    tr = Trainer(cfg, device="cpu", log=logs.append)
    tr.initialize()
    if rank == crash_rank:
        step = tr.train_step

        def crashing(*a, **k):
            if tr.metrics.step >= crash_after:
                raise _Crash()
            return step(*a, **k)

        tr.train_step = crashing
        try:
            tr.start_training()
        except _Crash:
            tr.membership.stop()  # no graceful leave: the heartbeat just stops
            tr.egroup.pg.abort()
            crashed_at = tr.metrics.step
            if not rejoin:
                return {"crashed_at": crashed_at}
        # the same rank restarts as a new process would: a fresh trainer that joins the running job,
        # once its old entry has aged out of the room (later still when the ring should re-form first)
        time.sleep(max(cfg.dead_after_s + 1, join_delay_s))
        logs = []
        tr = Trainer(apply_overrides(cfg, ["elastic_join=true"]), device="cpu", log=logs.append)
        tr.initialize()
    try:
        m = tr.start_training()
    except RuntimeError as e:
        tr.destroy()
        return {"error": str(e), "logs": logs}
    params = np.concatenate([v.detach().numpy().ravel() for v in tr.model.named().values()])
    tr.destroy()
    return {"step": m.step, "world": tr.world, "rank": tr.rank, "skipped": m.skipped_steps, "params": params,
            "logs": logs, "val_bpb": m.val_bpb}


def test_survivors_reform_the_ring_and_finish_in_lockstep():
    r0, r1, r2 = run_world(_elastic, 3, 2, 3, timeout=180)
    assert r2 == {"crashed_at": 3}
    for r in (r0, r1):
        assert r["step"] == 8 and r["world"] == 2 and r["skipped"] == 1, {k: r[k] for k in ("step", "world", "skipped")}
        assert np.isfinite(r["val_bpb"]) and r["val_bpb"] > 0
    assert (r0["rank"], r1["rank"]) == (0, 1)
    assert np.array_equal(r0["params"], r1["params"])
    assert any("ring re-formed: version 2, 2 peers" in line for line in r0["logs"]), r0["logs"]


def test_ring_below_min_size_stops_instead_of_training_on():
    r0, r1, r2 = run_world(_elastic, 3, 2, 3, ("min_ring_size=3", "reform_timeout_s=8"), timeout=180)
    assert r2 == {"crashed_at": 3}
    for r in (r0, r1):
        assert "ring stayed below min_ring_size=3" in r.get("error", ""), r
    assert any("ring too small (2/3)" in line for line in r0["logs"])


def test_restarted_rank_rejoins_a_paused_ring():
    """min_ring_size=3: the two survivors pause; the crashed rank's restart joins the room, the ring of
    three re-forms, the joiner receives the state from a survivor and all three finish identically."""
    r0, r1, r2 = run_world(_elastic, 3, 2, 3, ("min_ring_size=3",), True, timeout=240)
    for r in (r0, r1, r2):
        assert "error" not in r, r.get("error")
        assert r["step"] == 8 and r["world"] == 3, {k: r[k] for k in ("step", "world")}
    assert np.array_equal(r0["params"], r1["params"]) and np.array_equal(r0["params"], r2["params"])
    assert any(line.startswith("joined the ring at step") for line in r2["logs"]), r2["logs"]


def test_running_ring_takes_in_a_joiner():
    """min_ring_size=1: the survivors keep training as a ring of two; the restarted rank joins the room
    after that ring formed, and the running ring takes it in at its next check, after which all three
    train in lock-step."""
    r0, r1, r2 = run_world(_elastic, 3, 2, 3, ("join_check_steps=1", "max_steps=24"), True, 14.0, timeout=300)
    for r in (r0, r1, r2):
        assert "error" not in r, r.get("error")
        assert r["step"] == 24 and r["world"] == 3, {k: r[k] for k in ("step", "world")}
    assert np.array_equal(r0["params"], r1["params"]) and np.array_equal(r0["params"], r2["params"])
    assert any("ring re-formed: version 2, 2 peers" in line for line in r0["logs"]), r0["logs"]
    assert any("taking in ['rank00002-join" in line for line in r0["logs"]), r0["logs"][-5:]
    joined = [line for line in r2["logs"] if line.startswith("joined the ring at step")]
    assert joined and 4 < int(joined[0].split()[5].rstrip(":")) < 24, joined
