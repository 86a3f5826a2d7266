"""Coordinator of the centralised mode: hands out batches, collects per-worker loss statistics, runs
the step clock and serves status over REST and a dashboard WebSocket.

Behaviour follows the reference's coordinator (server/index.ts):

* a worker joins over the ``/ws`` WebSocket and gets ``WELCOME`` with the model config and batch size
  (:150-186); a round starts ``start_delay_s`` after a join (:182-185);
* a round gives every idle worker a ``BATCH_ASSIGN`` of synthetic data (:238-262); the reference's data
  is uniform random ids with independent uniform random targets (:81-97), ``data="reference"`` here;
  any data source of the trainer (``zipf``, ``markov``, ``uniform``, ``tokens``) can be used instead,
  one seeded stream per worker slot;
* a worker answers with ``GRADIENT_PUSH`` (loss, tokens processed, compute time); the coordinator does
  not aggregate gradients (:206-228); the step completes when every worker of the round has reported, or
  after ``straggler_timeout_s`` (30 s) with whoever did (:264-272);
* step completion averages the losses, keeps a debiased EMA (beta 0.9), the best loss, the token count
  and ``tokens/s = tokens / mean compute time`` (:275-329), broadcasts ``LOSS_UPDATE`` and
  ``STATUS_UPDATE`` to dashboards (:349-381) and starts the next round after ``next_round_delay_s``;
* REST: ``GET /api/status`` and ``GET /api/losses`` (:385-408); ``/data`` serves the prepared data
  directory (:57); shutdown sends ``KICK`` to every worker (:425-432).

Deliberate differences, each a defect of the reference's flow:

* the straggler timer belongs to its step; the reference's timer is never cleared, so a timer of an
  earlier round can complete a later round early;
* a join while a round is open does not start another round (the reference starts one per join, so
  rounds overlap); the new worker gets a batch in the next round;
* completion counts the workers the round was handed to and that are still connected: a worker that
  leaves mid-round completes the step at once instead of after the timeout, and a worker that joined
  mid-round is not waited for;
* a push for an earlier step is ignored instead of counted toward the current one;
* the EMA starts from 0 before debiasing (the reference starts it at the first loss and then debiases
  as well, which reports 10x the loss at step 1).
"""
from __future__ import annotations

import asyncio
import math
import os
import threading
import time
from dataclasses import dataclass, field

import numpy as np

from .protocol import MessageType, decode, encode_batch, encode_json


@dataclass
class CoordinatorConfig:
    host: str = "127.0.0.1"
    port: int = 8787  # 0 picks a free port
    batch_size: int = 0  # 0: the model preset's device batch
    data: str = "reference"
    straggler_timeout_s: float = 30.0
    start_delay_s: float = 2.0
    next_round_delay_s: float = 0.1
    min_workers: int = 1  # workers to wait for before the first round
    max_steps: int = 0  # 0: until stopped
    binary_batches: bool = True
    seed: int = 0
    data_dir: str = os.path.join("public", "data")
    linger_s: float = 0.0  # REST stays up this long after the last step (workers are kicked at once)


@dataclass
class WorkerInfo:
    id: str
    ws: object
    slot: int
    state: str = "idle"  # idle | training | disconnected
    device_info: dict = field(default_factory=dict)
    last_seen: float = 0.0
    joined_at: float = 0.0
    steps_completed: int = 0
    total_compute_ms: float = 0.0
    memory_usage: float = 0.0

    @property
    def device(self) -> str:
        d = self.device_info or {}
        return f"{d.get('vendor', '?')} {d.get('architecture', '')}".strip()


def model_config_message(model) -> dict:
    """``WELCOME.config`` fields (protocol.ts:57-65) from a :class:`GPTConfig`."""
    return {"sequenceLen": model.sequence_len, "vocabSize": model.vocab_size, "nLayer": model.n_layer,
            "nHead": model.n_head, "nKvHead": model.n_kv_head, "nEmbd": model.n_embd,
            "windowPattern": model.window_pattern}


class Coordinator:
    def __init__(self, cfg: CoordinatorConfig, train_cfg=None, log=print):
        from ..config import preset
        self.cfg = cfg
        self.train_cfg = train_cfg if train_cfg is not None else preset("ref-default")
        self.model_cfg = self.train_cfg.model
        self.batch_size = cfg.batch_size or self.train_cfg.device_batch
        self.log = log
        self.workers: dict[str, WorkerInfo] = {}
        self.dashboards: set = set()
        self.step = 0
        self.total_tokens = 0
        self.start_time = time.time()
        self.losses: list[float] = []
        self.ema = 0.0
        self.smooth_loss = 0.0
        self.best_loss = math.inf
        self.pending: dict[str, dict] = {}
        self.round_workers: set[str] = set()
        self.round_open = False
        self.timeouts = 0
        self.gradient_bytes = 0
        self._timer = None
        self._start_handle = None
        self._next_slot = 0
        self._sources: dict[int, object] = {}
        self.finished: asyncio.Event | None = None
        self.loop: asyncio.AbstractEventLoop | None = None
        self._runner = None
        self.port = cfg.port

    # ------------------------------------------------------------------ data
    def _batch(self, slot: int) -> tuple[np.ndarray, np.ndarray]:
        B, T, V = self.batch_size, self.model_cfg.sequence_len, self.model_cfg.vocab_size
        if self.cfg.data == "reference":
            rng = np.random.default_rng((self.cfg.seed, self.step, slot))
            return (rng.integers(0, V, size=(B, T), dtype=np.int32),
                    rng.integers(0, V, size=(B, T), dtype=np.int32))
        src = self._sources.get(slot)
        if src is None:
            import copy

            from ..data.pipeline import make_batch_source
            tc = copy.deepcopy(self.train_cfg)
            tc.data = self.cfg.data
            src = self._sources[slot] = make_batch_source(tc, "train", slot, 1)
        x, y = src.next(B, T)
        return np.ascontiguousarray(x, dtype=np.int32), np.ascontiguousarray(y, dtype=np.int32)

    # ------------------------------------------------------------------ messaging
    async def _send(self, ws, msg) -> None:
        try:
            if isinstance(msg, (bytes, bytearray)):
                await ws.send_bytes(bytes(msg))
            else:
                await ws.send_str(encode_json(msg))
        except (ConnectionError, RuntimeError):
            pass  # the close handler retires the worker

    async def _broadcast(self, msg: dict) -> None:
        for ws in list(self.dashboards):
            await self._send(ws, msg)

    def _worker_list(self) -> list[dict]:
        return [{"id": w.id, "state": w.state, "device": w.device, "lastSeen": w.last_seen,
                 "stepsCompleted": w.steps_completed,
                 "avgComputeTimeMs": w.total_compute_ms / w.steps_completed if w.steps_completed else 0.0,
                 "joinedAt": w.joined_at} for w in self.workers.values()]

    def status(self) -> dict:
        elapsed = time.time() - self.start_time
        return {"step": self.step, "loss": self.smooth_loss,
                "bestLoss": self.best_loss if math.isfinite(self.best_loss) else None,
                "numWorkers": len(self.workers), "tokensPerSec": self.total_tokens / max(elapsed, 1.0),
                "totalTokens": self.total_tokens, "elapsedSeconds": elapsed,
                "workers": [{k: w[k] for k in ("id", "state", "device", "stepsCompleted")} for w in self._worker_list()],
                "config": model_config_message(self.model_cfg), "timeouts": self.timeouts}

    async def _status_update(self) -> None:
        s = self.status()
        await self._broadcast({"type": int(MessageType.STATUS_UPDATE), "step": s["step"], "loss": s["loss"],
                               "bestLoss": s["bestLoss"], "numWorkers": s["numWorkers"],
                               "tokensPerSec": s["tokensPerSec"], "elapsedSeconds": s["elapsedSeconds"],
                               "totalTokens": s["totalTokens"], "workers": self._worker_list(),
                               "losses": self.losses[-100:]})

    # ------------------------------------------------------------------ worker messages
    async def on_join(self, ws, msg: dict) -> WorkerInfo:
        wid = str(msg.get("workerId") or f"worker-{self._next_slot}")
        now = time.time()
        w = WorkerInfo(wid, ws, self._next_slot, device_info=msg.get("deviceInfo") or {}, last_seen=now, joined_at=now)
        self._next_slot += 1
        self.workers[wid] = w
        self.log(f"[central] worker {wid} joined ({w.device or 'unknown device'}); {len(self.workers)} connected")
        await self._send(ws, {"type": int(MessageType.WELCOME), "workerId": wid,
                              "config": model_config_message(self.model_cfg), "batchSize": self.batch_size,
                              "totalWorkers": len(self.workers)})
        await self._status_update()
        if (not self.round_open and self._start_handle is None
                and (self.step > 0 or len(self.workers) >= self.cfg.min_workers)):
            self._start_handle = self.loop.call_later(self.cfg.start_delay_s, self._spawn, self.start_round())
        return w

    def on_heartbeat(self, msg: dict) -> None:
        w = self.workers.get(str(msg.get("workerId")))
        if w is not None:
            w.last_seen = time.time()
            w.memory_usage = float(msg.get("memoryUsage") or 0.0)

    async def on_push(self, msg: dict) -> None:
        w = self.workers.get(str(msg.get("workerId")))
        if w is None:
            return
        w.last_seen = time.time()
        if not self.round_open or int(msg.get("stepId", -1)) != self.step or w.id not in self.round_workers:
            return  # a push for an earlier round
        w.steps_completed += 1
        w.total_compute_ms += float(msg.get("computeTimeMs") or 0.0)
        w.state = "idle"
        self.pending[w.id] = {"loss": float(msg.get("loss", math.nan)),
                              "tokensProcessed": int(msg.get("tokensProcessed") or 0),
                              "computeTimeMs": float(msg.get("computeTimeMs") or 0.0)}
        await self._maybe_complete()

    async def on_leave(self, wid: str, reason: str) -> None:
        w = self.workers.pop(wid, None)
        if w is None:
            return
        w.state = "disconnected"
        self.log(f"[central] worker {wid} {reason}; {len(self.workers)} remaining")
        await self._status_update()
        await self._maybe_complete()

    # ------------------------------------------------------------------ rounds
    def _spawn(self, coro) -> None:
        self._start_handle = None
        asyncio.ensure_future(coro)

    async def start_round(self) -> None:
        if self.round_open or (self.finished is not None and self.finished.is_set()):
            return
        idle = [w for w in self.workers.values() if w.state == "idle"]
        # min_workers gates the first round only; later rounds run with whoever is connected
        if len(idle) < (max(1, self.cfg.min_workers) if self.step == 0 else 1):
            return  # the next join starts it
        self.step += 1
        self.pending.clear()
        self.round_workers = {w.id for w in idle}
        self.round_open = True
        for w in idle:
            x, y = self._batch(w.slot)
            w.state = "training"
            if self.cfg.binary_batches:
                await self._send(w.ws, encode_batch(self.step, x, y))
            else:
                await self._send(w.ws, {"type": int(MessageType.BATCH_ASSIGN), "stepId": self.step,
                                        "inputIds": x.ravel().astype(np.uint32), "targets": y.ravel()})
        await self._status_update()
        step = self.step
        self._timer = self.loop.call_later(self.cfg.straggler_timeout_s, self._on_timeout, step)

    def _on_timeout(self, step: int) -> None:
        if self.round_open and step == self.step:
            expected = len(self.round_workers & set(self.workers))
            self.log(f"[central] step {step}: timeout, {len(self.pending)}/{expected} workers reported")
            self.timeouts += 1
            asyncio.ensure_future(self.complete_step())

    async def _maybe_complete(self) -> None:
        if not self.round_open:
            return
        expected = self.round_workers & set(self.workers)
        if set(self.pending) >= expected:
            await self.complete_step()

    async def complete_step(self) -> None:
        if not self.round_open:
            return
        self.round_open = False
        if self._timer is not None:
            self._timer.cancel()
            self._timer = None
        for wid in self.round_workers:  # stragglers become idle again and get the next round's batch
            w = self.workers.get(wid)
            if w is not None:
                w.state = "idle"
        if self.pending:
            n = len(self.pending)
            loss = sum(p["loss"] for p in self.pending.values()) / n
            tokens = sum(p["tokensProcessed"] for p in self.pending.values())
            compute_ms = sum(p["computeTimeMs"] for p in self.pending.values()) / n
            beta = 0.9
            self.ema = beta * self.ema + (1 - beta) * loss
            self.smooth_loss = self.ema / (1 - beta ** len(self.losses + [loss]))
            self.total_tokens += tokens
            self.losses.append(loss)
            self.best_loss = min(self.best_loss, loss)
            elapsed = time.time() - self.start_time
            tps = tokens / (compute_ms / 1000.0) if compute_ms > 0 else 0.0
            self.log(f"[central] step {self.step} complete | loss={self.smooth_loss:.6f} | {n} workers | "
                     f"{tps:.0f} tok/s | {elapsed:.0f}s")
            await self._broadcast({"type": int(MessageType.LOSS_UPDATE), "step": self.step, "loss": loss,
                                   "smoothLoss": self.smooth_loss, "bestLoss": self.best_loss, "numWorkers": n,
                                   "tokensPerSec": tps, "totalTokens": self.total_tokens, "elapsed": elapsed})
        else:
            self.log(f"[central] step {self.step}: no worker reported")
        await self._status_update()
        self.pending.clear()
        if self.cfg.max_steps and self.step >= self.cfg.max_steps:
            self.finished.set()
            return
        self.loop.call_later(self.cfg.next_round_delay_s, self._spawn, self.start_round())

    # ------------------------------------------------------------------ transport
    def app(self):
        from aiohttp import WSMsgType, web

        async def ws_handler(request):
            ws = web.WebSocketResponse(max_msg_size=0)
            await ws.prepare(request)
            if "dashboard" in request.query_string or "dashboard" in request.path:
                self.dashboards.add(ws)
                await self._status_update()
                try:
                    async for _ in ws:
                        pass
                finally:
                    self.dashboards.discard(ws)
                return ws
            wid = None
            try:
                async for m in ws:
                    if m.type not in (WSMsgType.TEXT, WSMsgType.BINARY):
                        continue
                    try:
                        msg = decode(m.data)
                    except Exception as e:  # a malformed frame is logged and dropped (index.ts:123-130)
                        self.log(f"[central] bad frame: {e}")
                        continue
                    t = int(msg.get("type", 0))
                    if t == MessageType.WORKER_JOIN:
                        wid = (await self.on_join(ws, msg)).id
                    elif t == MessageType.WORKER_HEARTBEAT:
                        self.on_heartbeat(msg)
                    elif t == MessageType.GRADIENT_PUSH:
                        if "data" in msg:  # a binary gradient frame: counted, not aggregated
                            self.gradient_bytes += int(msg["data"].nbytes)
                        else:
                            await self.on_push(msg)
                    elif t == MessageType.WORKER_LEAVE:
                        await self.on_leave(str(msg.get("workerId", wid)), "left")
                        wid = None
            finally:
                if wid is not None:
                    await self.on_leave(wid, "disconnected")
            return ws

        async def status(_request):
            return web.json_response(self.status())

        async def losses(_request):
            return web.json_response({"losses": self.losses})

        app = web.Application()
        app.router.add_get("/ws", ws_handler)
        app.router.add_get("/api/status", status)
        app.router.add_get("/api/losses", losses)
        if os.path.isdir(self.cfg.data_dir):
            app.router.add_static("/data", self.cfg.data_dir)
        return app

    async def start(self) -> int:
        """Binds the server; returns the port."""
        from aiohttp import web
        self.loop = asyncio.get_running_loop()
        self.finished = asyncio.Event()
        self._runner = web.AppRunner(self.app())
        await self._runner.setup()
        site = web.TCPSite(self._runner, self.cfg.host, self.cfg.port)
        await site.start()
        self.port = site._server.sockets[0].getsockname()[1]
        self.start_time = time.time()
        self.log(f"[central] coordinator on http://{self.cfg.host}:{self.port} (ws /ws, /api/status); model "
                 f"{self.model_cfg.n_layer}L/{self.model_cfg.n_embd}D/{self.model_cfg.n_head}H, vocab "
                 f"{self.model_cfg.vocab_size}, seq {self.model_cfg.sequence_len}, batch {self.batch_size}")
        return self.port

    async def shutdown(self) -> None:
        for w in list(self.workers.values()):
            await self._send(w.ws, {"type": int(MessageType.KICK)})
        if self.cfg.linger_s > 0:
            await asyncio.sleep(self.cfg.linger_s)
        for ws in list(self.dashboards):
            await ws.close()
        if self._runner is not None:
            await self._runner.cleanup()

    async def serve(self) -> None:
        """Runs until ``max_steps`` rounds completed (or forever), then kicks the workers."""
        await self.start()
        try:
            await self.finished.wait()
        finally:
            await self.shutdown()


class CoordinatorThread:
    """Runs a :class:`Coordinator` on its own event loop in a background thread (tests, notebooks)."""

    def __init__(self, coord: Coordinator):
        self.coord = coord
        self.loop = asyncio.new_event_loop()
        self._ready = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        asyncio.set_event_loop(self.loop)
        try:
            self.loop.run_until_complete(self.coord.start())
            self._ready.set()
            self.loop.run_until_complete(self.coord.finished.wait())
            self.loop.run_until_complete(self.coord.shutdown())
        finally:
            self.loop.close()

    def start(self) -> int:
        self.thread.start()
        if not self._ready.wait(30):
            raise RuntimeError("coordinator did not start")
        return self.coord.port

    def stop(self, timeout: float = 30.0) -> None:
        if self.coord.finished is not None:
            self.loop.call_soon_threadsafe(self.coord.finished.set)
        self.thread.join(timeout)

    def call(self, fn):
        """Runs ``fn()`` on the coordinator's loop and returns its result."""
        import concurrent.futures
        fut: concurrent.futures.Future = concurrent.futures.Future()

        def run():
            try:
                fut.set_result(fn())
            except BaseException as e:
                fut.set_exception(e)

        self.loop.call_soon_threadsafe(run)
        return fut.result(30)
