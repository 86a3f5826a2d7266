"""Centralised mode on one B200: a coordinator on 127.0.0.1 and workers on cuda:0, one training a
128-wide-head model through the sm_100a engine, one the reference's 4 x 64 default through the eager
path."""
import asyncio
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(train_cfg, steps, data):
    from bitresearch_b200.central import CentralWorker, Coordinator, CoordinatorConfig, CoordinatorThread
    logs = []
    coord = Coordinator(CoordinatorConfig(port=0, start_delay_s=0.2, max_steps=steps, straggler_timeout_s=120,
                                          data=data), train_cfg, log=logs.append)
    th = CoordinatorThread(coord)
    port = th.start()
    out = {}

    def go():
        w = CentralWorker(f"ws://127.0.0.1:{port}/ws", device="cuda:0", worker_id="gpu0", log=lambda m: None)
        out["res"] = asyncio.run(w.run())
        out["impl"] = w.trainer.cfg.impl if w.trainer is not None else None

    t = threading.Thread(target=go, daemon=True)
    t.start()
    t.join(300)
    th.thread.join(60)
    return coord, out


def test_central_worker_on_engine(cuda):
    from bitresearch_b200.config import apply_overrides, preset
    tc = apply_overrides(preset("d512"), ["model.n_layer=2", "model.n_embd=256", "model.n_head=2",
                                          "model.n_kv_head=2", "model.sequence_len=512", "device_batch=4"])
    coord, out = _run(tc, 6, "markov")
    assert out["res"]["steps"] == 6 and out["impl"] == "cuda"
    assert coord.step == 6 and np.isfinite(coord.losses).all() and coord.losses[-1] < coord.losses[0]


def test_central_worker_reference_default_on_engine(cuda):
    """The reference's default model (4 x 64 heads) trains on the sm_100a engine."""
    from bitresearch_b200.config import preset
    coord, out = _run(preset("ref-default"), 2, "reference")
    assert out["res"]["steps"] == 2 and out["impl"] == "cuda"
    assert np.isfinite(coord.losses).all()
