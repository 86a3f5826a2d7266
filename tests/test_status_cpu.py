"""Job status over HTTP: the trainer's and the swarm's GET /status (the reference signalling server's
fields) and GET /metrics (Prometheus text)."""
import json
import urllib.request

import pytest

pytest.importorskip("aiohttp")

from bitresearch_b200.config import apply_overrides, preset  # noqa: E402
from bitresearch_b200.utils.status import StatusServer, prometheus_text  # noqa: E402


def _get(url):
    with urllib.request.urlopen(url, timeout=10) as r:
        return r.read().decode()


def test_prometheus_text_skips_non_numbers():
    t = prometheus_text("x", {"step": 3, "loss": 1.5, "name": "a", "nan": float("nan"), "flag": True,
                              "extra": {"val_bpb_floor": 0.4}})
    assert "# TYPE x_step gauge\nx_step 3\n" in t and "x_loss 1.5" in t and "x_extra_val_bpb_floor 0.4" in t
    assert "name" not in t and "x_nan" not in t and "x_flag" not in t


def test_trainer_serves_status_and_metrics():
    from bitresearch_b200.train import Trainer
    cfg = apply_overrides(preset("tiny-cpu"), ["model.n_layer=1", "model.n_embd=64", "model.n_head=1",
                                               "model.n_kv_head=1", "model.sequence_len=32", "model.vocab_size=128",
                                               "device_batch=2", "total_batch_tokens=64", "eval_tokens=128",
                                               "log_every=1", "results_tsv=", "max_steps=3", "status_port=0"])
    tr = Trainer(cfg, device="cpu", log=lambda m: None)
    tr.initialize()
    tr.start_training()
    base = tr.status_server.url
    st = json.loads(_get(base + "/status"))
    assert st["totalPeers"] == 1 and st["computePeers"] == 1 and st["rooms"] == ["default"]
    assert st["peers"][0]["position"] == 0 and st["training"]["step"] == 3 and st["training"]["val_bpb"] > 0
    m = _get(base + "/metrics")
    assert "bitresearch_step 3" in m and "bitresearch_val_bpb" in m
    assert tr.status_server.published == 3 + 1  # metrics on every logging step (log_every=1) + completion
    tr.destroy()
    assert tr.status_server is None


def test_swarm_queue_status_and_server():
    from bitresearch_b200.swarm.runner import SwarmQueue
    q = SwarmQueue([{"id": i, "description": f"v{i}"} for i in range(7)], chunk_size=3)
    q.next_chunk("w0")
    q.record({"params": {"id": 1, "description": "v1"}, "metrics": {"sharpe": 0.7}})
    q.record({"params": {"id": 0, "description": "v0"}, "metrics": {"sharpe": 1.2}})
    s = q.status()
    assert (s["totalVariants"], s["completed"], s["results"], s["bestScore"]) == (7, 2, 2, 1.2)
    srv = StatusServer(lambda: {"swarms": {"swarm": q.status()}}, q.status, prefix="sw")
    srv.start()
    try:
        assert json.loads(_get(srv.url + "/status"))["swarms"]["swarm"]["completed"] == 2
        assert "sw_bestScore 1.2" in _get(srv.url + "/metrics")
    finally:
        srv.stop()


def test_observer_feed_receives_published_messages():
    import asyncio
    import threading
    import time

    import aiohttp
    srv = StatusServer(lambda: {})
    srv.start()
    got = []

    async def observe():
        async with aiohttp.ClientSession() as s, s.ws_connect(srv.url.replace("http", "ws") + "/ws") as ws:
            async for m in ws:
                got.append(json.loads(m.data))

    t = threading.Thread(target=lambda: asyncio.run(observe()), daemon=True)
    t.start()
    deadline = time.time() + 10
    while srv.subscribers < 1:
        assert time.time() < deadline
        time.sleep(0.02)
    for i in range(3):
        srv.publish({"type": "swarm-progress", "totalCompleted": i + 1, "totalVariants": 3})
    srv.publish({"type": "swarm-complete", "results": []})
    srv.stop()  # delivers what was published first
    t.join(10)
    assert [m["type"] for m in got] == ["swarm-progress"] * 3 + ["swarm-complete"]
    assert got[2]["totalCompleted"] == 3


def test_swarm_emits_progress_and_completion_events():
    from bitresearch_b200.swarm.runner import run_swarm
    from bitresearch_b200.swarm.strategy import synthetic_market, variant_grid
    events = []
    res = run_swarm(variant_grid()[:4], synthetic_market(), workers=1, n_paths=300, log=lambda m: None,
                    on_event=events.append)
    prog = [e for e in events if e["type"] == "swarm-progress"]
    assert len(res) == 4 and len(prog) == 4 and prog[-1]["totalCompleted"] == 4 and prog[-1]["totalVariants"] == 4
    assert all(e["result"]["params"]["id"] in range(4) and e["peerId"] == "worker-0" for e in prog)
    assert events[-1]["type"] == "swarm-complete" and len(events[-1]["results"]) == 4
