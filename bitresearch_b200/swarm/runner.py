"""Swarm work queue: independent strategy variants farmed out in chunks to worker processes.

The reference runs this as a side mode of its signalling server (server/signaling.ts:306-405): the
server holds the variant list, hands each compute peer the next chunk of ``chunkSize`` (5) unassigned,
uncompleted variants, records results as they arrive, keeps them sorted by Sharpe, broadcasts progress
(completed / total, best score and variant) and gives the reporting peer its next chunk until the list
is exhausted. Here the coordinator is a process-local object and the peers are worker processes (one
per GPU, or CPU workers), talking over multiprocessing queues. One deliberate difference: variants
assigned to a worker that exits before reporting them are put back in the queue (the reference keeps
them assigned, so they would never complete).

  python -m bitresearch_b200.swarm [--workers N] [--paths 50000] [--variants config.json]
                                   [--data val.json] [--out results.json] [--status-port P]
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import queue
import sys
import time


class SwarmQueue:
    """Chunk assignment and result bookkeeping (the server side of the swarm)."""

    def __init__(self, variants: list[dict], chunk_size: int = 5):
        self.variants = variants
        self.chunk_size = chunk_size
        self.completed: set[int] = set()
        self.assigned: dict[int, str] = {}  # variant index -> worker
        self.results: list[dict] = []
        self.start = time.time()

    def next_chunk(self, worker: str) -> list[dict]:
        nxt = next((i for i in range(len(self.variants)) if i not in self.completed and i not in self.assigned), -1)
        if nxt < 0:
            return []
        picked = [i for i in range(nxt, min(nxt + self.chunk_size, len(self.variants)))
                  if i not in self.completed and i not in self.assigned]
        for i in picked:
            self.assigned[i] = worker
        return [self.variants[i] for i in picked]

    def record(self, result: dict) -> dict:
        vid = result.get("params", {}).get("id")
        if vid is None:
            return {}
        idx = next((i for i, v in enumerate(self.variants) if v.get("id") == vid), None)
        if idx is not None:
            self.completed.add(idx)
            self.assigned.pop(idx, None)
        self.results.append(result)
        self.results.sort(key=lambda r: -(r.get("metrics", {}).get("sharpe", 0.0)))
        best = self.results[0]
        return {"totalCompleted": len(self.completed), "totalVariants": len(self.variants),
                "bestScore": best["metrics"].get("sharpe", 0.0), "bestVariant": best["params"].get("description", "")}

    def release(self, worker: str) -> int:
        """Puts a departed worker's unfinished variants back in the queue; returns how many."""
        lost = [i for i, w in self.assigned.items() if w == worker]
        for i in lost:
            del self.assigned[i]
        return len(lost)

    @property
    def done(self) -> bool:
        return len(self.completed) >= len(self.variants)

    def status(self) -> dict:
        """Progress in the signalling server's ``swarms`` form (server/signaling.ts:142-151)."""
        best = self.results[0]["metrics"].get("sharpe") if self.results else None
        return {"totalVariants": len(self.variants), "completed": len(self.completed), "results": len(self.results),
                "bestScore": best, "elapsedMs": (time.time() - self.start) * 1e3}


def _worker(name: str, device: str | None, data: dict, n_paths: int, seed: int, req_q, work_q, res_q) -> None:
    from .strategy import run_variant
    if device and device.startswith("cuda"):
        import torch
        torch.cuda.set_device(torch.device(device))
    req_q.put(("request", name))
    while True:
        chunk = work_q.get()
        if chunk is None:
            return
        for v in chunk:
            t0 = time.time()
            try:
                r = run_variant(v, data, n_paths=n_paths, seed=seed, device=device)
            except Exception as e:  # a crashing variant scores -9, as in the reference
                r = {"params": v, "metrics": {"sharpe": -9, "calmar": -9, "max_drawdown": -1, "win_rate": 0,
                                               "total_return": -1, "sharpe_ci_low": -9, "sharpe_ci_high": -9,
                                               "mc_mean_sharpe": -9, "mc_std_sharpe": 0}, "error": str(e)}
            r["peerId"] = name
            r["elapsedMs"] = round((time.time() - t0) * 1000)
            res_q.put(("result", name, r))
        req_q.put(("request", name))


def run_swarm(variants: list[dict], data: dict, workers: int = 1, n_paths: int = 50_000, seed: int = 0,
              devices: list[str] | None = None, chunk_size: int = 5, log=print, timeout_s: float = 3600.0,
              status_port: int = -1, on_event=None) -> list[dict]:
    """Runs every variant on ``workers`` processes; returns the results sorted by Sharpe (best first).
    ``status_port >= 0`` serves the progress at ``GET /status`` and ``GET /metrics`` meanwhile and pushes
    ``swarm-progress`` / ``swarm-complete`` to ``/ws`` observers (server/signaling.ts:380-400); ``on_event``
    receives the same messages in-process."""
    ctx = mp.get_context("spawn")
    q = SwarmQueue(variants, chunk_size)
    server = None
    if status_port >= 0:
        from ..utils.status import StatusServer
        t0 = time.time() * 1e3

        def status():
            peers = [{"id": f"worker-{w}", "room": "swarm", "position": w, "peerType": "compute", "joinedAt": t0}
                     for w in range(workers)]
            return {"rooms": ["swarm"], "peers": peers, "ringVersion": 0, "totalPeers": workers,
                    "computePeers": workers, "observerPeers": 0, "swarms": {"swarm": q.status()}}

        server = StatusServer(status, q.status, port=status_port, prefix="bitresearch_swarm")
        server.start()
        log(f"[swarm] status: {server.url}/status, observers: {server.url.replace('http', 'ws')}/ws")

    def emit(msg: dict) -> None:
        if server is not None:
            server.publish(msg)
        if on_event is not None:
            on_event(msg)

    req_q, res_q = ctx.Queue(), ctx.Queue()
    work_qs, procs = {}, {}
    devices = devices or [None] * workers
    for w in range(workers):
        name = f"worker-{w}"
        work_qs[name] = ctx.Queue()
        p = ctx.Process(target=_worker, args=(name, devices[w % len(devices)], data, n_paths, seed, req_q,
                                              work_qs[name], res_q), daemon=True)
        p.start()
        procs[name] = p
    deadline = time.time() + timeout_s
    idle: set[str] = set()
    try:
        while not q.done and time.time() < deadline:
            try:
                kind, name, *rest = res_q.get(timeout=0.05)
                prog = q.record(rest[0])
                log(f"[swarm] {prog['totalCompleted']}/{prog['totalVariants']} best sharpe {prog['bestScore']:.4f} "
                    f"({prog['bestVariant']})")
                emit({"type": "swarm-progress", **prog, "result": rest[0], "peerId": name})
            except queue.Empty:
                pass
            while True:
                try:
                    kind, name = req_q.get_nowait()
                except queue.Empty:
                    break
                chunk = q.next_chunk(name)
                if chunk:
                    work_qs[name].put(chunk)
                    idle.discard(name)
                else:
                    idle.add(name)
            for name, p in list(procs.items()):
                if not p.is_alive() and p.exitcode not in (0, None):
                    n = q.release(name)
                    log(f"[swarm] {name} exited ({p.exitcode}); {n} variants requeued")
                    del procs[name]
            if idle and not q.done:  # work freed up by a departed worker goes to an idle one
                for name in list(idle):
                    chunk = q.next_chunk(name)
                    if chunk and name in procs:
                        work_qs[name].put(chunk)
                        idle.discard(name)
            if not procs:
                raise RuntimeError("all swarm workers exited")
        if q.done:
            emit({"type": "swarm-complete", "results": q.results[:20]})
    finally:
        for name, wq in work_qs.items():
            wq.put(None)
        for p in procs.values():
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
        if server is not None:
            server.stop()
    if not q.done:
        raise TimeoutError(f"swarm finished {len(q.completed)} of {len(variants)} variants before the deadline")
    return q.results


def main(argv=None) -> int:
    from .strategy import MC_PATHS, synthetic_market, variant_grid
    ap = argparse.ArgumentParser(description="strategy swarm: RSI variants with Monte-Carlo Sharpe intervals")
    ap.add_argument("--workers", type=int, default=0, help="worker processes (default: one per GPU, else 1)")
    ap.add_argument("--paths", type=int, default=MC_PATHS)
    ap.add_argument("--variants", default="", help="config.json with a 'variants' list (default: the built-in grid)")
    ap.add_argument("--data", default="", help="json {ticker: [closes] or {close: [...]}} (default: synthetic)")
    ap.add_argument("--limit", type=int, default=0, help="only the first N variants")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--out", default="")
    ap.add_argument("--status-port", type=int, default=-1, help=">= 0: serve GET /status and /metrics")
    args = ap.parse_args(argv)
    import torch
    ngpu = torch.cuda.device_count()
    workers = args.workers or max(ngpu, 1)
    devices = [f"cuda:{i}" for i in range(ngpu)] if ngpu else [None]
    if args.variants:
        with open(args.variants) as f:
            variants = json.load(f)["variants"]
    else:
        variants = variant_grid()
    if args.limit:
        variants = variants[:args.limit]
    if args.data:
        with open(args.data) as f:
            raw = json.load(f)
        data = {k: (v["close"] if isinstance(v, dict) else v) for k, v in raw.items()}
    else:
        data = synthetic_market(seed=args.seed)
    t0 = time.time()
    results = run_swarm(variants, data, workers=workers, n_paths=args.paths, seed=args.seed, devices=devices,
                        status_port=args.status_port)
    print(f"[swarm] {len(results)} variants in {time.time() - t0:.1f}s on {workers} worker(s)")
    for i, r in enumerate(results[:15]):
        m = r["metrics"]
        print(f"{i + 1:3d} sharpe {m['sharpe']:8.4f} mc {m['mc_mean_sharpe']:8.4f} "
              f"[{m['sharpe_ci_low']:.3f}, {m['sharpe_ci_high']:.3f}] dd {m['max_drawdown']:.4f}  "
              f"{r['params']['description']}")
    if args.out:
        with open(args.out, "w") as f:
            json.dump(results, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
