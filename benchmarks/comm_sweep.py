"""Reduce-scatter / all-reduce sweep: the in-kernel NVLink collectives against NCCL.

  timeout -k 60 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \
      --master-addr 127.0.0.1 --master-port 29511 benchmarks/comm_sweep.py [--json out.jsonl]

Bucket sizes 1 KB .. 256 MB (powers of 4) of N(0,1) values from a seed, for every rank. Variants:

* ``nccl_rs`` / ``nccl_ar``: ``reduce_scatter_tensor`` / ``all_reduce`` (ReduceOp.AVG) on a tensor of the
  wire dtype (fp32, bf16 or fp16).
* ``p2p_rs_push``: the trainer's path for one bucket: ``comm_pack_push`` (fp32 -> wire dtype and the
  non-finite check fused; each owner's slice is stored into that owner's receive slot for this rank,
  posted NVLink stores), ``comm_signal_all`` (one release flag per owner) and ``comm_reduce_local``
  (each owner sums its N slots from local memory, fp32, 1/N).
* ``p2p_rs``: the pull form: ``comm_pack`` into this rank's own buffer, a release flag, and
  ``comm_reduce`` where each owner reads its slice from every peer's buffer over NVLink.
* ``p2p_ar``: ``p2p_rs`` into a symmetric result buffer, then every owner pushes its reduced slice
  (fp32) into each peer's buffer with posted NVLink stores (``comm_push``), the pair the trainer runs
  per step (gradient reduce-scatter, parameter push).
* ``p2p_topk``: top-k (1%) select with error feedback fused into the (u32 index, f16 value) list
  writer, and the owners' sparse merge (``topk_reduce``); compared against the dense rows.

The reference's counterpart is the WebRTC ring all-reduce (ring-allreduce.ts:85-215) with an f16
wire (webrtc-mesh.ts:551-577). Times are CUDA-event device times per iteration, the max over ranks.
Bus bandwidth follows the NCCL convention: reduce-scatter moves (N-1)/N of the bucket per rank,
all-reduce 2(N-1)/N; the roofline is the measured 770 GB/s per direction peer copy (900 nominal).
Our own iterations include the flag waits that make buffer reuse safe (a rank repacks its send buffer
only after every peer has finished reading the previous iteration's data).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

LINK_GBS = 770.0  # measured peer copy bandwidth per direction on this B200 pool (900 nominal)
WIRE = {"fp32": (0, torch.float32, 4), "bf16": (1, torch.bfloat16, 2), "fp16": (2, torch.float16, 2)}
SLOT_READY, SLOT_READ, SLOT_RES, SLOT_GATHERED = 0, 1, 2, 3


class P2PBench:
    """Symmetric buffers for the largest size, plus the flag protocol of one iteration."""

    def __init__(self, max_elems: int, rank: int, world: int, budget_s: float = 10.0):
        from bitresearch_b200.ops._ext import ext
        from bitresearch_b200.parallel.comm import SymmetricBuffer
        self.E = ext()
        self.rank, self.world = rank, world
        self.budget = budget_s
        self.send = SymmetricBuffer(max_elems * 4)
        self.recv = SymmetricBuffer(max_elems * 4 + 64 * world)
        self.rflags = SymmetricBuffer(world * 8)
        self.recv_peers = torch.tensor(self.recv.peer_ptrs, dtype=torch.int64, device="cuda")
        self.rflag_peers = torch.tensor(self.rflags.peer_ptrs, dtype=torch.int64, device="cuda")
        self.res = SymmetricBuffer(max_elems * 4)
        self.flags = SymmetricBuffer(64 * 8)
        self.push_flags = SymmetricBuffer(world * 8)
        self.no_segs = torch.zeros(0, 7, dtype=torch.int64, device="cuda")
        self.idx = SymmetricBuffer(max_elems * 4)
        self.val = SymmetricBuffer(max_elems * 2)
        self.cnt = SymmetricBuffer(64 * 4)
        self.flag_ptrs = torch.tensor(self.flags.peer_ptrs, dtype=torch.int64, device="cuda")
        self.res_view = self.res.view(max_elems, 0)
        self.cnt_view = self.cnt.view(64, 0)
        self.sp_peers = torch.tensor([[self.idx.peer_ptrs[r], self.val.peer_ptrs[r], self.cnt.peer_ptrs[r]]
                                      for r in range(world)], dtype=torch.int64, device="cuda")
        self.empty = torch.zeros(1, 2, dtype=torch.int64, device="cuda")
        self.dummy = torch.zeros(8, device="cuda")
        self.bad = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.epoch = 0
        self.last = {}  # slot -> last epoch this rank signalled (every rank runs the same sequence)

    def setup(self, n: int, chunk: int = 1 << 15):
        """Ownership of an n-element bucket: rank r owns [r*n/N, (r+1)*n/N)."""
        from bitresearch_b200.parallel.comm import chunk_ranges, interleave_by_owner
        W, r = self.world, self.rank
        per = n // W
        self.n, self.per = n, per
        rows = [(o, ln) for o, ln, _ in chunk_ranges(r * per, per, size=chunk)]
        self.chunks = torch.tensor(rows, dtype=torch.int64, device="cuda").view(-1, 2)
        push = [(o * per + s, ln, o, s) for o in range(W) for _, ln, s in chunk_ranges(o * per, per, size=chunk)]
        self.push_tab = torch.tensor(interleave_by_owner(push, r, W), dtype=torch.int64, device="cuda").view(-1, 4)
        self.own_tab = torch.tensor([t for t in push if t[2] == r], dtype=torch.int64, device="cuda").view(-1, 4)
        segs = []
        for o in range(W):
            if o != r:
                for off, ln, _ in chunk_ranges(o * per, per, size=chunk):
                    segs.append((off, ln, o, 0, 0, 0, 0))
        self.segs = torch.tensor(segs, dtype=torch.int64, device="cuda").view(-1, 7)
        sel = []
        for o in range(W):
            for off, ln, _ in chunk_ranges(o * per, per, size=1 << 14):
                sel.append((off, ln, o * per, o))
        self.sel = torch.tensor(sel, dtype=torch.int64, device="cuda").view(-1, 4)
        self.err = torch.zeros(n, device="cuda")
        self.thr = torch.zeros(1, device="cuda")
        self.blocks = min(len(rows), 2 * torch.cuda.get_device_properties(0).multi_processor_count)

    def _wait(self, slot: int):
        """Waits until every peer has signalled ``slot`` as often as this rank has."""
        epoch = self.last.get(slot, 0)
        if epoch > 0:
            self.E.comm_reduce(self.send.peers_dev, self.flag_ptrs, slot, epoch, self.empty, self.dummy, 0, 1.0, 1,
                               self.budget)

    def _signal(self, slot: int, epoch: int):
        self.E.comm_signal(self.flags.ptr + 8 * slot, epoch)
        self.last[slot] = epoch

    def rs(self, src: torch.Tensor, wire: int, out: torch.Tensor, mark=None):
        mark = mark or (lambda name: None)
        e = self.epoch = self.epoch + 1
        self._wait(SLOT_READ)  # every peer has read last iteration's send buffer
        mark("wait_read")
        self.E.comm_pack(src, self.send.ptr, wire, 0, self.n, 1.0, self.bad)
        mark("pack")
        self._signal(SLOT_READY, e)
        mark("signal")
        self.E.comm_reduce(self.send.peers_dev, self.flag_ptrs, SLOT_READY, e, self.chunks, out, wire,
                           1.0 / self.world, self.blocks, self.budget)
        mark("reduce")
        self._signal(SLOT_READ, e)

    def rs_push(self, src: torch.Tensor, wire: int, out: torch.Tensor):
        e = self.epoch = self.epoch + 1
        self._wait(SLOT_READ)  # every owner has summed last iteration's slots
        self.E.comm_pack_push(src, self.recv_peers, self.rank, self.per, self.push_tab, wire, 1.0, self.bad,
                              self.blocks)
        self.E.comm_signal_all(self.rflag_peers, self.rank, 0, e, self.bad)
        self.E.comm_reduce_local(self.recv.ptr, self.rflags.ptr, self.world, 0, e, self.per, self.own_tab, out, wire,
                                 1.0 / self.world, self.blocks, self.budget)
        self._signal(SLOT_READ, e)

    def ar(self, src: torch.Tensor, wire: int, mark=None):
        """Reduce-scatter, then each owner pushes its reduced slice into every peer's result buffer
        (posted NVLink stores) and flags them; a rank is done when all owners' flags arrived."""
        mark = mark or (lambda name: None)
        e = self.epoch + 1
        self._wait(SLOT_GATHERED)  # every peer has consumed last iteration's result
        mark("wait_gathered")
        self.rs(src, wire, self.res_view, mark)
        self.E.comm_push(self.res_view, self.res.peers_dev, self.rank, self.chunks, self.blocks)
        self.E.comm_signal_peers(self.push_flags.peers_dev, self.rank, e)
        mark("push")
        self.E.comm_shadow_refresh(self.res_view, self.push_flags.ptr, self.world, self.rank, e, self.no_segs, 1,
                                   self.budget)
        mark("wait_pushes")
        self._signal(SLOT_GATHERED, e)
        mark("signal3")

    def topk(self, src: torch.Tensor, ratio: float, out: torch.Tensor):
        e = self.epoch = self.epoch + 1
        self._wait(SLOT_READ)  # every peer has read last iteration's lists and counters
        self.cnt_view.zero_()
        self.E.topk_threshold(src, self.err, None, 0, self.n, 1.0, 0.0, 10000, ratio, e * 7919 + self.rank, False, self.thr)
        self.E.topk_select(src, self.err, None, self.sel, 1.0, 0.0, False, self.thr, self.idx.ptr, self.val.ptr, self.cnt.ptr)
        self._signal(SLOT_READY, e)
        out[self.rank * self.per:(self.rank + 1) * self.per].zero_()
        self.E.topk_reduce(self.sp_peers, self.flag_ptrs, SLOT_READY, e, self.rank * self.per, self.rank, out,
                           1.0 / self.world, self.blocks, self.budget)
        self._signal(SLOT_READ, e)

    def close(self):
        for b in (self.send, self.recv, self.rflags, self.res, self.flags, self.push_flags, self.idx, self.val,
                  self.cnt):
            b.close()


def time_iters(fn, iters: int, warm: int = 3) -> float:
    """Per-iteration device time (ms), max over ranks."""
    for _ in range(warm):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    dist.barrier()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def breakdown(bench: P2PBench, nbytes: int, wire: str, iters: int = 20) -> dict:
    """Device time of each phase of one p2p all-reduce iteration (median over iterations, max over ranks)."""
    code, _, esz = WIRE[wire]
    n = max(8 * bench.world, (nbytes // esz) // (8 * bench.world) * (8 * bench.world))
    bench.setup(n)
    src = torch.randn(n, device="cuda")
    rows = []
    for it in range(iters + 3):
        evs = []

        def mark(name, evs=evs):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            evs.append((name, ev))

        mark("start")
        bench.ar(src, code, mark)
        torch.cuda.synchronize()
        if it >= 3:
            rows.append({evs[i][0]: evs[i - 1][1].elapsed_time(evs[i][1]) * 1e3 for i in range(1, len(evs))})
    out = {}
    for k in rows[0]:
        vals = sorted(r[k] for r in rows)
        t = torch.tensor([vals[len(vals) // 2]], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[k] = round(float(t.item()), 2)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-bytes", type=int, default=1 << 10)
    ap.add_argument("--max-bytes", type=int, default=256 << 20)
    ap.add_argument("--wires", default="fp32,bf16,fp16")
    ap.add_argument("--variants", default="nccl_rs,p2p_rs_push,p2p_rs,nccl_ar,p2p_ar,p2p_topk")
    ap.add_argument("--topk", type=float, default=0.01)
    ap.add_argument("--json", default="")
    ap.add_argument("--breakdown", default="", help="comma-separated bucket sizes (bytes): per-phase us of p2p_ar")
    args = ap.parse_args()

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from bitresearch_b200.ops._ext import check_status

    sizes = []
    s = args.min_bytes
    while s <= args.max_bytes:
        sizes.append(s)
        s *= 4
    max_elems = args.max_bytes // 2 + 8 * world
    bench = P2PBench(max_elems, rank, world)
    variants = args.variants.split(",")
    if args.breakdown:
        for nb in args.breakdown.split(","):
            for wname in args.wires.split(","):
                ph = breakdown(bench, int(nb), wname)
                if rank == 0:
                    print(json.dumps({"breakdown_us": ph, "bytes": int(nb), "wire": wname, "n_gpus": world}), flush=True)
    rows = []
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    for wname in args.wires.split(","):
        code, dt, esz = WIRE[wname]
        for nbytes in sizes:
            n = max(8 * world, (nbytes // esz) // (8 * world) * (8 * world))
            src32 = torch.randn(n, device="cuda", generator=gen)
            src = src32.to(dt)
            bench.setup(n)
            red = torch.zeros(n, device="cuda")
            iters = 50 if nbytes <= (1 << 20) else 20 if nbytes <= (16 << 20) else 8
            for v in variants:
                if v == "p2p_topk" and wname != "fp16":
                    continue  # one top-k row per size: f16 values on the wire
                if v == "nccl_rs":
                    out = torch.empty(n // world, dtype=dt, device="cuda")
                    fn = lambda: dist.reduce_scatter_tensor(out, src, op=dist.ReduceOp.AVG)  # noqa: E731
                elif v == "nccl_ar":
                    buf = src.clone()
                    fn = lambda: dist.all_reduce(buf, op=dist.ReduceOp.AVG)  # noqa: E731
                elif v == "p2p_rs":
                    fn = lambda: bench.rs(src32, code, red)  # noqa: E731
                elif v == "p2p_rs_push":
                    fn = lambda: bench.rs_push(src32, code, red)  # noqa: E731
                elif v == "p2p_ar":
                    fn = lambda: bench.ar(src32, code)  # noqa: E731
                elif v == "p2p_topk":
                    fn = lambda: bench.topk(src32, args.topk, red)  # noqa: E731
                else:
                    raise SystemExit(f"unknown variant {v}")
                ms = time_iters(fn, iters)
                st = check_status()
                flag = torch.tensor([st], device="cuda")
                dist.all_reduce(flag, op=dist.ReduceOp.MAX)
                factor = (world - 1) / world * (2 if v.endswith("_ar") else 1)
                bus = n * esz * factor / (ms * 1e-3) / 1e9
                row = {"variant": v, "wire": wname, "bytes": n * esz, "n_gpus": world, "us": round(ms * 1e3, 2),
                       "busbw_gbs": round(bus, 1), "frac_of_link": round(bus / LINK_GBS, 3),
                       "status": int(flag.item())}
                if v == "p2p_topk":
                    row["note"] = f"top-{args.topk:g} of an fp32 bucket; busbw is dense-equivalent"
                rows.append(row)
                if rank == 0:
                    print(json.dumps(row), flush=True)
    dist.barrier()
    torch.cuda.synchronize()
    bench.close()
    if rank == 0 and args.json:
        with open(args.json, "w") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
