"""Centralised mode on CPU: protocol codecs, a coordinator with CPU workers over WebSockets on
127.0.0.1, the straggler timeout, departures mid-round, stale pushes, REST and the dashboard feed."""
import asyncio
import json
import threading
import time
import urllib.request

import numpy as np
import pytest

aiohttp = pytest.importorskip("aiohttp")

from bitresearch_b200.central import (CentralWorker, Coordinator, CoordinatorConfig, CoordinatorThread,  # noqa: E402
                                      MessageType, decode, encode_batch, encode_json, encode_tensor_message)
from bitresearch_b200.config import preset  # noqa: E402


def test_protocol_round_trips():
    msg = {"type": 3, "workerId": "w", "gradients": np.arange(5, dtype=np.float32),
           "ids": np.array([1, 2], dtype=np.uint32), "t": np.array([-1, 7], dtype=np.int32), "loss": 1.5}
    text = encode_json(msg)
    assert '"__typed_array": true' in text and '"type": "Float32Array"' in text
    back = decode(text)
    assert back["gradients"].dtype == np.float32 and back["ids"].dtype == np.uint32 and back["t"].dtype == np.int32
    assert back["t"].tolist() == [-1, 7] and back["loss"] == 1.5
    # tensor frame: u8 type | u32 step | u32 count, data at byte 12
    buf = encode_tensor_message(MessageType.PARAMS_BROADCAST, 7, np.array([1.0, -2.0], np.float32))
    assert len(buf) == 12 + 8 and buf[0] == 0x11 and int.from_bytes(buf[1:5], "little") == 7
    assert int.from_bytes(buf[5:9], "little") == 2 and np.frombuffer(buf[12:], "<f4").tolist() == [1.0, -2.0]
    t = decode(buf)
    assert t["type"] == 0x11 and t["stepId"] == 7 and t["data"].tolist() == [1.0, -2.0]
    x = np.arange(12, dtype=np.int32).reshape(3, 4)
    b = decode(encode_batch(5, x, x + 1))
    assert b["type"] == MessageType.BATCH_ASSIGN and b["stepId"] == 5
    assert np.array_equal(b["inputIds"], x) and np.array_equal(b["targets"], x + 1)


def _tiny():
    tc = preset("tiny-cpu")
    tc.device_batch = 2
    return tc


def _run_workers(port, n, **kw):
    results, threads = [None] * n, []

    def go(i):
        w = CentralWorker(f"ws://127.0.0.1:{port}/ws", device="cpu", worker_id=f"cpu-{i}", log=lambda m: None, **kw)
        results[i] = asyncio.run(w.run())

    for i in range(n):
        t = threading.Thread(target=go, args=(i,), daemon=True)
        t.start()
        threads.append(t)
    return results, threads


def _get(port, path):
    with urllib.request.urlopen(f"http://127.0.0.1:{port}{path}", timeout=10) as r:
        return json.loads(r.read())


def test_coordinator_with_two_cpu_workers_and_dashboard():
    logs = []
    coord = Coordinator(CoordinatorConfig(port=0, start_delay_s=0.3, max_steps=4, min_workers=2,
                                          straggler_timeout_s=60), _tiny(), log=logs.append)
    th = CoordinatorThread(coord)
    port = th.start()
    feed = []

    async def dashboard():
        async with aiohttp.ClientSession() as s, s.ws_connect(f"http://127.0.0.1:{port}/ws?dashboard=1") as ws:
            async for m in ws:
                feed.append(json.loads(m.data))

    dt = threading.Thread(target=lambda: asyncio.run(dashboard()), daemon=True)
    dt.start()
    time.sleep(0.2)
    st = _get(port, "/api/status")
    assert st["step"] == 0 and st["config"]["nLayer"] == 2 and st["config"]["sequenceLen"] == 128
    results, threads = _run_workers(port, 2)
    for t in threads:
        t.join(120)
    assert all(r is not None and r["kicked"] and r["steps"] == 4 for r in results), results
    th.thread.join(30)
    assert coord.step == 4 and len(coord.losses) == 4 and coord.timeouts == 0
    assert all(np.isfinite(coord.losses)) and coord.total_tokens == 4 * 2 * 2 * 128
    # standard debiased EMA: the first smoothed value is the first loss itself
    ema = 0.0
    for i, l in enumerate(coord.losses):
        ema = 0.9 * ema + 0.1 * l
    assert abs(coord.smooth_loss - ema / (1 - 0.9 ** 4)) < 1e-9
    kinds = [m["type"] for m in feed]
    assert MessageType.STATUS_UPDATE in kinds and kinds.count(MessageType.LOSS_UPDATE) == 4
    first = next(m for m in feed if m["type"] == MessageType.LOSS_UPDATE)
    assert abs(first["smoothLoss"] - first["loss"]) < 1e-9 and first["numWorkers"] == 2


def test_rest_endpoints_and_json_batches():
    coord = Coordinator(CoordinatorConfig(port=0, start_delay_s=0.2, max_steps=2, binary_batches=False,
                                          straggler_timeout_s=60, linger_s=5.0), _tiny(), log=lambda m: None)
    th = CoordinatorThread(coord)
    port = th.start()
    results, threads = _run_workers(port, 1)
    deadline = time.time() + 60
    while not coord.finished.is_set():
        assert time.time() < deadline
        time.sleep(0.05)
    losses = _get(port, "/api/losses")["losses"]
    st = _get(port, "/api/status")
    assert len(losses) == 2 and st["step"] == 2 and st["totalTokens"] == 2 * 2 * 128
    for t in threads:
        t.join(60)
    th.thread.join(30)
    assert results[0]["steps"] == 2


async def _fake_worker(port, on_batch):
    async with aiohttp.ClientSession() as s, s.ws_connect(f"http://127.0.0.1:{port}/ws", max_msg_size=0) as ws:
        await ws.send_str(encode_json({"type": 1, "workerId": "fake", "deviceInfo": {"vendor": "test"}}))
        async for m in ws:
            msg = decode(m.data)
            if msg["type"] == MessageType.BATCH_ASSIGN:
                if await on_batch(ws, msg) == "close":
                    return
            elif msg["type"] == MessageType.KICK:
                return


def test_straggler_timeout_and_stale_pushes():
    logs = []
    coord = Coordinator(CoordinatorConfig(port=0, start_delay_s=0.2, max_steps=2, min_workers=2,
                                          straggler_timeout_s=3.0), _tiny(), log=logs.append)
    th = CoordinatorThread(coord)
    port = th.start()

    async def stale(ws, msg):  # never reports this step; reports an older one instead
        await ws.send_str(encode_json({"type": 3, "workerId": "fake", "stepId": msg["stepId"] - 1, "loss": 99.0,
                                       "tokensProcessed": 1, "computeTimeMs": 1.0}))

    ft = threading.Thread(target=lambda: asyncio.run(_fake_worker(port, stale)), daemon=True)
    ft.start()
    results, threads = _run_workers(port, 1)
    for t in threads + [ft]:
        t.join(90)
    th.thread.join(30)
    assert coord.step == 2 and coord.timeouts == 2
    assert len(coord.losses) == 2 and max(coord.losses) < 50  # the stale 99.0 never counted
    assert sum("timeout, 1/2 workers reported" in l for l in logs) == 2


def test_departure_mid_round_completes_without_waiting():
    logs = []
    coord = Coordinator(CoordinatorConfig(port=0, start_delay_s=0.2, max_steps=2, min_workers=2,
                                          straggler_timeout_s=120.0), _tiny(), log=logs.append)
    th = CoordinatorThread(coord)
    port = th.start()

    async def leave(ws, msg):
        return "close"

    ft = threading.Thread(target=lambda: asyncio.run(_fake_worker(port, leave)), daemon=True)
    ft.start()
    t0 = time.time()
    results, threads = _run_workers(port, 1)
    for t in threads + [ft]:
        t.join(90)
    th.thread.join(30)
    assert coord.step == 2 and coord.timeouts == 0 and time.time() - t0 < 60
    assert any("fake disconnected" in l for l in logs)


def test_worker_config_follows_welcome_and_engine_support():
    from bitresearch_b200.central.worker import train_config_from_welcome
    from bitresearch_b200.central.coordinator import model_config_message
    from bitresearch_b200.models.engine import FusedGPTEngine
    ref = preset("ref-default")
    assert FusedGPTEngine.unsupported(ref.model) is None  # 4 x 64 heads run on the engine too
    assert FusedGPTEngine.unsupported(preset("d512").model) is None
    odd = preset("ref-default").model
    odd.n_head, odd.n_kv_head = 8, 8  # 32-wide heads: eager path
    assert FusedGPTEngine.unsupported(odd) is not None
    welcome = {"config": model_config_message(ref.model), "batchSize": 3}
    c = train_config_from_welcome(welcome, "cpu")
    assert (c.model.n_layer, c.model.n_embd, c.model.n_head, c.model.sequence_len) == (4, 256, 4, 512)
    assert c.device_batch == 3 and c.total_batch_tokens == 3 * 512 and c.impl == "torch" and c.dtype == "fp32"
    assert train_config_from_welcome(welcome, "cuda:0").impl == "cuda"  # the engine runs 64-wide heads
    d = preset("d512")
    assert train_config_from_welcome({"config": model_config_message(d.model), "batchSize": 2}, "cuda:0").impl == "cuda"


def test_local_mode_spawns_workers_and_finishes():
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-m", "bitresearch_b200.central", "local", "--preset", "tiny-cpu",
                          "--max-steps", "2", "--start-delay", "0.3", "--port", "0", "--workers", "2"],
                         capture_output=True, text=True, timeout=240, cwd=root,
                         env={**os.environ, "PYTHONUNBUFFERED": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    assert "step 2 complete" in out.stdout and "2 workers" in out.stdout
    assert out.stdout.count("'kicked': True") == 2
