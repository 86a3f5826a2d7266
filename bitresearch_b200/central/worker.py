"""Worker of the centralised mode: one process per GPU (or a CPU process) that joins a coordinator,
trains its own model replica on the batches it is handed and reports loss statistics.

The protocol side follows src/distributed/protocol.ts (the reference's worker client is not in its
tree; its messages are): ``WORKER_JOIN`` with device info, ``WORKER_HEARTBEAT`` every few seconds with
the memory in use, one ``GRADIENT_PUSH`` (loss, tokens processed, compute time) per ``BATCH_ASSIGN``,
``WORKER_LEAVE`` on a clean exit, and exit on ``KICK``. The coordinator does not aggregate gradients,
so each worker steps its own optimizer (MuonAdamW through the sm_100a engine on a GPU, the torch path on
CPU). ``push_gradients=True`` also sends the flat gradient as a binary tensor frame before the
statistics, like the reference's ``gradients`` field; the coordinator only counts its bytes.

All torch work runs on one executor thread, so the event loop keeps answering (heartbeats, kicks)
during a step.
"""
from __future__ import annotations

import asyncio
import concurrent.futures
import os
import time
import uuid

import numpy as np

from .protocol import MessageType, decode, encode_json, encode_tensor_message


def device_info(device: str) -> dict:
    import torch
    if device.startswith("cuda") and torch.cuda.is_available():
        p = torch.cuda.get_device_properties(torch.device(device))
        return {"vendor": "NVIDIA", "architecture": f"sm_{p.major}{p.minor}", "description": p.name,
                "maxBufferSize": int(p.total_memory)}
    return {"vendor": "cpu", "architecture": os.uname().machine, "description": "host CPU", "maxBufferSize": 0}


def train_config_from_welcome(msg: dict, device: str):
    """The worker's :class:`TrainConfig`: the coordinator's model and batch, one micro-batch per step."""
    from ..config import preset
    c = msg["config"]
    cfg = preset("ref-default")
    m = cfg.model
    m.sequence_len, m.vocab_size = int(c["sequenceLen"]), int(c["vocabSize"])
    m.n_layer, m.n_head, m.n_kv_head, m.n_embd = int(c["nLayer"]), int(c["nHead"]), int(c["nKvHead"]), int(c["nEmbd"])
    m.window_pattern = str(c["windowPattern"])
    cfg.device_batch = int(msg["batchSize"])
    cfg.total_batch_tokens = cfg.device_batch * m.sequence_len
    cfg.results_tsv, cfg.log_every, cfg.data = "", 0, "uniform"
    if not device.startswith("cuda"):
        cfg.impl, cfg.dtype, cfg.ns_dtype = "torch", "fp32", "fp32"
    else:
        from ..models.engine import FusedGPTEngine
        # the sm_100a engine when it supports the model (64- and 128-wide heads), else the eager path on the GPU
        cfg.impl = "cuda" if FusedGPTEngine.unsupported(m) is None else "torch"
    return cfg


class CentralWorker:
    def __init__(self, url: str, device: str | None = None, worker_id: str | None = None, heartbeat_s: float = 5.0,
                 push_gradients: bool = False, log=print):
        import torch
        self.url = url
        self.device = device or ("cuda:0" if torch.cuda.is_available() else "cpu")
        self.worker_id = worker_id or f"worker-{uuid.uuid4().hex[:12]}"
        self.heartbeat_s = heartbeat_s
        self.push_gradients = push_gradients
        self.log = log
        self.trainer = None
        self.steps = 0
        self.last_loss = float("nan")
        self.kicked = False
        self._pool = concurrent.futures.ThreadPoolExecutor(max_workers=1)

    # ------------------------------------------------------------------ torch side (executor thread)
    def _build(self, welcome: dict) -> None:
        import torch
        from ..train import Trainer
        if self.device.startswith("cuda"):
            torch.cuda.set_device(torch.device(self.device))
        self.trainer = Trainer(train_config_from_welcome(welcome, self.device), device=self.device,
                               log=lambda m: None)
        self.trainer.initialize()

    def _train(self, x: np.ndarray, y: np.ndarray):
        import torch
        t0 = time.perf_counter()
        dev = self.trainer.device
        xt = torch.from_numpy(np.array(x, dtype=np.int32)).to(dev)  # frames decode to read-only views
        yt = torch.from_numpy(np.array(y, dtype=np.int32)).to(dev)
        loss = float(self.trainer.train_step(batch=(xt, yt)))
        ms = (time.perf_counter() - t0) * 1e3
        grad = self.trainer.flat_grad.detach().float().cpu().numpy() if self.push_gradients else None
        return loss, ms, grad

    def _memory(self) -> float:
        import torch
        if self.device.startswith("cuda") and torch.cuda.is_available():
            return float(torch.cuda.memory_allocated(torch.device(self.device)))
        return 0.0

    # ------------------------------------------------------------------ protocol side
    async def _heartbeat(self, ws) -> None:
        while not ws.closed:
            await asyncio.sleep(self.heartbeat_s)
            if ws.closed:
                return
            await ws.send_str(encode_json({"type": int(MessageType.WORKER_HEARTBEAT), "workerId": self.worker_id,
                                           "timestamp": time.time() * 1e3, "memoryUsage": self._memory()}))

    async def run(self, max_steps: int = 0) -> dict:
        """Serves batches until kicked, disconnected or ``max_steps`` pushes were sent (then leaves)."""
        import aiohttp
        loop = asyncio.get_running_loop()
        info = await loop.run_in_executor(self._pool, device_info, self.device)
        async with aiohttp.ClientSession() as session:
            async with session.ws_connect(self.url, max_msg_size=0) as ws:
                await ws.send_str(encode_json({"type": int(MessageType.WORKER_JOIN), "workerId": self.worker_id,
                                               "deviceInfo": info, "timestamp": time.time() * 1e3}))
                hb = asyncio.ensure_future(self._heartbeat(ws))
                try:
                    async for m in ws:
                        if m.type not in (aiohttp.WSMsgType.TEXT, aiohttp.WSMsgType.BINARY):
                            continue
                        msg = decode(m.data)
                        t = int(msg.get("type", 0))
                        if t == MessageType.WELCOME:
                            await loop.run_in_executor(self._pool, self._build, msg)
                            self.log(f"[worker {self.worker_id}] joined: {msg['config']} batch {msg['batchSize']}")
                        elif t == MessageType.BATCH_ASSIGN and self.trainer is not None:
                            T = self.trainer.cfg.model.sequence_len
                            x = np.asarray(msg["inputIds"]).reshape(-1, T)
                            y = np.asarray(msg["targets"]).reshape(-1, T)
                            loss, ms, grad = await loop.run_in_executor(self._pool, self._train, x, y)
                            self.steps += 1
                            self.last_loss = loss
                            if grad is not None:
                                await ws.send_bytes(encode_tensor_message(MessageType.GRADIENT_PUSH, msg["stepId"], grad))
                            await ws.send_str(encode_json({
                                "type": int(MessageType.GRADIENT_PUSH), "workerId": self.worker_id,
                                "stepId": int(msg["stepId"]), "loss": loss, "tokensProcessed": int(x.size),
                                "computeTimeMs": ms}))
                            if max_steps and self.steps >= max_steps:
                                await ws.send_str(encode_json({"type": int(MessageType.WORKER_LEAVE),
                                                               "workerId": self.worker_id}))
                                break
                        elif t == MessageType.KICK:
                            self.kicked = True
                            break
                finally:
                    hb.cancel()
        if self.trainer is not None:
            await loop.run_in_executor(self._pool, self.trainer.destroy)
        self._pool.shutdown(wait=True)
        return {"workerId": self.worker_id, "steps": self.steps, "loss": self.last_loss, "kicked": self.kicked}


def run_worker_process(url: str, device: str | None, max_steps: int = 0, push_gradients: bool = False,
                       cpu_threads: int = 0) -> None:
    """Entry point of one worker process (an importable target for ``multiprocessing``). ``cpu_threads``
    caps torch's intra-op threads, so CPU workers sharing a host do not oversubscribe its cores."""
    if cpu_threads > 0:
        import torch
        torch.set_num_threads(cpu_threads)
    w = CentralWorker(url, device=device, push_gradients=push_gradients)
    res = asyncio.run(w.run(max_steps=max_steps))
    print(f"[worker] {res}", flush=True)
