"""HTTP status of a running job: ``GET /status`` (JSON) and ``GET /metrics`` (Prometheus text format).

The reference's signalling server answers ``GET /status`` with its rooms, peers (id, room, ring
position, peer type, join time), ring version, peer counts and swarm progress (server/signaling.ts:
129-160). Here the training job itself serves the same fields (one room, one compute peer per rank, a
static ring: torch.distributed does not re-form the group), plus the trainer's metrics; the strategy
swarm serves its progress under ``swarms``. ``/metrics`` exposes the numeric fields as gauges for a
Prometheus scrape.

``/ws`` is a push feed for observers (the reference's observer page joins the swarm room and receives
``swarm-progress`` / ``swarm-complete`` messages, observer.html:50-80): every message given to
``publish`` goes to each connected client as JSON.

The server runs on its own event loop in a daemon thread and only reads what the providers return, so
the training loop never waits for it.
"""
from __future__ import annotations

import asyncio
import json
import math
import threading
from typing import Callable


def prometheus_text(prefix: str, values: dict) -> str:
    """``# TYPE <prefix>_<key> gauge`` + value lines for every finite number in ``values`` (one level of
    nesting is flattened with ``_``)."""
    lines = []
    flat = {}
    for k, v in values.items():
        if isinstance(v, dict):
            for k2, v2 in v.items():
                flat[f"{k}_{k2}"] = v2
        else:
            flat[k] = v
    for k, v in flat.items():
        if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v):
            continue
        name = f"{prefix}_{''.join(c if c.isalnum() else '_' for c in k)}"
        lines.append(f"# TYPE {name} gauge")
        lines.append(f"{name} {float(v):.10g}")
    return "\n".join(lines) + "\n"


class StatusServer:
    def __init__(self, status: Callable[[], dict], metrics: Callable[[], dict] | None = None,
                 host: str = "127.0.0.1", port: int = 0, prefix: str = "bitresearch"):
        self.status_fn, self.metrics_fn = status, metrics or status
        self.host, self.port, self.prefix = host, port, prefix
        self.loop = asyncio.new_event_loop()
        self._ready = threading.Event()
        self._stop: asyncio.Event | None = None
        self._error: BaseException | None = None
        self._subs: set = set()
        self._pending: set = set()
        self.published = 0
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _app(self):
        from aiohttp import web

        async def status(_req):
            return web.Response(text=json.dumps(self.status_fn(), default=str), content_type="application/json",
                                headers={"Access-Control-Allow-Origin": "*"})

        async def metrics(_req):
            return web.Response(text=prometheus_text(self.prefix, self.metrics_fn()),
                                content_type="text/plain")

        async def feed(request):
            ws = web.WebSocketResponse()
            await ws.prepare(request)
            self._subs.add(ws)
            try:
                async for _ in ws:
                    pass
            finally:
                self._subs.discard(ws)
            return ws

        app = web.Application()
        app.router.add_get("/status", status)
        app.router.add_get("/metrics", metrics)
        app.router.add_get("/ws", feed)
        return app

    async def _broadcast(self, text: str) -> None:
        for ws in list(self._subs):
            try:
                await ws.send_str(text)
            except (ConnectionError, RuntimeError):
                self._subs.discard(ws)

    def publish(self, msg: dict) -> None:
        """Sends ``msg`` to every ``/ws`` client; callable from any thread, never blocks."""
        if self._stop is None or not self.thread.is_alive() or self.loop.is_closed():
            return
        text = json.dumps(msg, default=str)
        self.published += 1

        def start():
            task = asyncio.ensure_future(self._broadcast(text))
            self._pending.add(task)
            task.add_done_callback(self._pending.discard)

        self.loop.call_soon_threadsafe(start)

    async def _drain_and_stop(self) -> None:
        if self._pending:
            await asyncio.wait(list(self._pending), timeout=5)
        self._stop.set()

    @property
    def subscribers(self) -> int:
        return len(self._subs)

    def _run(self):
        from aiohttp import web
        asyncio.set_event_loop(self.loop)

        async def main():
            runner = web.AppRunner(self._app())
            await runner.setup()
            site = web.TCPSite(runner, self.host, self.port)
            await site.start()
            self.port = site._server.sockets[0].getsockname()[1]
            self._stop = asyncio.Event()
            self._ready.set()
            await self._stop.wait()
            await runner.cleanup()

        try:
            self.loop.run_until_complete(main())
        except BaseException as e:  # surfaced by start()
            self._error = e
            self._ready.set()
        finally:
            self.loop.close()

    @property
    def url(self) -> str:
        return f"http://{self.host}:{self.port}"

    def start(self) -> int:
        self.thread.start()
        self._ready.wait(30)
        if self._error is not None:
            raise RuntimeError(f"status server failed to start: {self._error}")
        return self.port

    def stop(self) -> None:
        """Delivers what was published, then shuts the server down."""
        if self._stop is not None and self.thread.is_alive():
            self.loop.call_soon_threadsafe(lambda: asyncio.ensure_future(self._drain_and_stop()))
            self.thread.join(10)
