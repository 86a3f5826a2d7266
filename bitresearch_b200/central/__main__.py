"""Command line of the centralised mode.

  python -m bitresearch_b200.central serve  [--port 8787] [--preset ref-default] [--data reference]
                                            [--max-steps N] [--straggler-timeout 30] [key=value ...]
  python -m bitresearch_b200.central worker --url ws://127.0.0.1:8787/ws [--device cuda:0] [--max-steps N]
  python -m bitresearch_b200.central local  [--workers N] [--max-steps N]   # coordinator + one worker per GPU
"""
from __future__ import annotations

import argparse
import asyncio
import multiprocessing as mp
import os
import sys


def _coordinator(args):
    from ..config import apply_overrides, preset
    from .coordinator import Coordinator, CoordinatorConfig
    tc = apply_overrides(preset(args.preset), list(args.overrides))
    cc = CoordinatorConfig(host=args.host, port=args.port, batch_size=args.batch_size, data=args.data,
                           straggler_timeout_s=args.straggler_timeout, start_delay_s=args.start_delay,
                           max_steps=args.max_steps, min_workers=args.min_workers,
                           binary_batches=not args.json_batches, data_dir=args.data_dir)
    return Coordinator(cc, tc)


def _serve_args(ap):
    ap.add_argument("--host", default="127.0.0.1")
    # PORT and BATCH_SIZE from the environment, as the reference's coordinator reads them (server/index.ts:42-43)
    ap.add_argument("--port", type=int, default=int(os.environ.get("PORT", "8787")))
    ap.add_argument("--preset", default="ref-default")
    ap.add_argument("--batch-size", type=int, default=int(os.environ.get("BATCH_SIZE", "0")))
    ap.add_argument("--data", default="reference", help="reference | zipf | markov | uniform | tokens")
    ap.add_argument("--straggler-timeout", type=float, default=30.0)
    ap.add_argument("--start-delay", type=float, default=2.0)
    ap.add_argument("--min-workers", type=int, default=1)
    ap.add_argument("--max-steps", type=int, default=0)
    ap.add_argument("--json-batches", action="store_true", help="send batches as JSON lists like the reference")
    ap.add_argument("--data-dir", default="public/data")
    ap.add_argument("overrides", nargs="*")




def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="centralised coordinator / worker")
    sub = ap.add_subparsers(dest="cmd", required=True)
    _serve_args(sub.add_parser("serve"))
    w = sub.add_parser("worker")
    w.add_argument("--url", default="ws://127.0.0.1:8787/ws")
    w.add_argument("--device", default=None)
    w.add_argument("--max-steps", type=int, default=0)
    w.add_argument("--push-gradients", action="store_true")
    loc = sub.add_parser("local")
    _serve_args(loc)
    loc.add_argument("--workers", type=int, default=0, help="default: one per GPU, else 1")
    args = ap.parse_args(argv)
    if args.cmd == "serve":
        asyncio.run(_coordinator(args).serve())
        return 0
    if args.cmd == "worker":
        from .worker import run_worker_process
        run_worker_process(args.url, args.device, args.max_steps, args.push_gradients)
        return 0
    import torch
    from .coordinator import CoordinatorThread
    n_gpu = torch.cuda.device_count()
    n = args.workers or max(1, n_gpu)
    args.min_workers = max(args.min_workers, n)
    args.port = args.port if args.port else 0
    th = CoordinatorThread(_coordinator(args))
    port = th.start()
    from .worker import run_worker_process
    ctx = mp.get_context("spawn")
    cpu_threads = 0 if n_gpu else max(1, (os.cpu_count() or 1) // n)
    procs = [ctx.Process(target=run_worker_process, args=(f"ws://{args.host}:{port}/ws",
                                                          f"cuda:{i % n_gpu}" if n_gpu else "cpu", 0, False,
                                                          cpu_threads))
             for i in range(n)]
    for p in procs:
        p.start()
    rc = 0
    try:
        while th.thread.is_alive():
            th.thread.join(1.0)
            if th.thread.is_alive() and not any(p.is_alive() for p in procs):
                print("[central] every worker process exited before the run finished", file=sys.stderr)
                th.stop()
                rc = 1
    except KeyboardInterrupt:
        th.stop()
    for p in procs:
        p.join(timeout=60)
    return rc


if __name__ == "__main__":
    sys.exit(main())
