"""Data-parallel gradient synchronisation with in-kernel NVLink collectives (one process per GPU).

Replaces the reference's WebRTC ring all-reduce (src/distributed/ring-allreduce.ts:85-215) on an
NVSwitch node with a direct algorithm:

* **Layout.** The trainer's flat fp32 gradient buffer is ordered by backward completion (lm_head,
  then layers L-1 .. 0, then embeddings/scalars), so each *bucket* (one layer's parameters) is one
  contiguous range. Parameters live in a symmetric (CUDA-IPC exported) fp32 buffer with the same
  offsets; gradients are packed into a symmetric send buffer in the wire dtype.
* **Ownership (sharded optimizer).** Every parameter tensor has one owner rank (greedy balance by
  size, Newton-Schulz work counted for matrices). Only the owner keeps optimizer state and updates it.
* **Per bucket, overlapped with backward** (comm stream, after an event recorded when the engine
  finishes the bucket), a push reduce-scatter: ``pack_push`` (fp32 -> wire dtype, 1/loss-scale,
  non-finite check; each parameter's slice is stored straight into its owner's receive slot for this
  rank, posted NVLink stores) -> ``signal_all`` (flags[bucket][me] = 2*step + non-finite bit on every
  rank, release) -> ``reduce_local`` (each owner waits on its local flags and sums the N slots from
  local memory in rank order, fp32, scaled by 1/N). No load crosses NVLink. The 1/N scale is the mean,
  fixing the reference's ring, which returns the sum (ring-allreduce.ts:161-165).
* **Skip agreement on the device:** after the last bucket, ``agree`` ORs the non-finite bits every rank
  sent with that bucket's flag (and the status word) into a device skip word, which the optimizer
  kernels read; the host never waits for the step. It learns the outcome one step later from a pinned
  copy (the reference's ``allReduce() -> null`` skip, without a host round trip).
* **After backward:** the sharded MuonAdamW step on owned parameters, then ``push``: each owner
  stores its updated parameters into every peer's symmetric parameter buffer with posted NVLink stores
  and flags each peer; each rank waits (bounded) for the other owners' flags and refreshes the bf16
  GEMM shadows of the parameters it does not own from its local copy. (``comm_gather`` is the pull
  form of the same exchange, kept for the collective sweep.)
* **Failure handling:** every device-side wait is bounded (``comm_timeout_s``); a timeout sets the
  device status word, the host sees it and reports the step as aborted (the reference's
  ``allReduce() -> null``). Non-finite gradients on any rank skip the update on all ranks.
"""
from __future__ import annotations

from collections import OrderedDict

import numpy as np
import torch
import torch.distributed as dist

from ..ops._ext import check_status, ext
from ..utils.timing import traced

WIRE_CODE = {"fp32": 0, "f32": 0, "bf16": 1, "fp16": 2, "f16": 2}
WIRE_BYTES = {0: 4, 1: 2, 2: 2}
ALIGN = 16  # elements; keeps every parameter 64-byte aligned in the flat buffers
CHUNK = 1 << 16
COMM_CTAS = 32  # CTAs per bucket kernel of the reduce-scatter


def bucket_order(specs, n_layer: int) -> list[list[str]]:
    """Parameter names grouped by the point in backward where their gradients are final."""
    names = [n for n, _, _ in specs]
    buckets = [["lmHead"]]
    for i in reversed(range(n_layer)):
        b = [n for n in names if n.startswith(f"layer{i}_")]
        if f"ve_{i}" in names:
            b.append(f"ve_{i}")
        buckets.append(b)
    buckets.append(["wte", "residLambdas", "x0Lambdas"])
    return buckets


def forward_groups(specs, n_layer: int) -> list[list[str]]:
    """Parameter names grouped by the point in the forward that first reads them: embeddings and the
    residual scalars, then each layer with its value embedding, then the lm_head. The parameter exchange
    after the sharded optimizer runs group by group in this order, so the next forward can start on
    the first groups while the later ones are still crossing NVLink."""
    names = [n for n, _, _ in specs]
    groups = [[n for n in ("wte", "residLambdas", "x0Lambdas") if n in names]]
    for i in range(n_layer):
        g = [n for n in names if n.startswith(f"layer{i}_")]
        if f"ve_{i}" in names:
            g.append(f"ve_{i}")
        groups.append(g)
    groups.append(["lmHead"])
    return groups


def flat_layout(specs, n_layer: int):
    """(OrderedDict name -> (offset, numel, shape), bucket ranges [(lo, hi)], bucket names, total)."""
    shapes = {n: s for n, s, _ in specs}
    layout: "OrderedDict[str, tuple[int, int, tuple]]" = OrderedDict()
    ranges, groups = [], bucket_order(specs, n_layer)
    off = 0
    for grp in groups:
        lo = off
        for n in grp:
            numel = int(np.prod(shapes[n]))
            layout[n] = (off, numel, tuple(shapes[n]))
            off += -(-numel // ALIGN) * ALIGN
        ranges.append((lo, off))
    return layout, ranges, groups, off


def assign_owners(specs, world: int) -> dict[str, int]:
    """Greedy longest-processing-time assignment of whole parameters to ranks.

    Cost = elements (optimizer memory traffic) plus, for matrices, the Newton-Schulz FLOPs expressed
    in element-equivalents, so the Muon work is spread too. Deterministic on every rank.
    """
    costs = []
    for n, shape, group in specs:
        numel = int(np.prod(shape))
        c = float(numel)
        if group == "matrices" and len(shape) == 2:
            r, cc = shape
            small, big = min(r, cc), max(r, cc)
            c += 15 * 2 * small * small * big / 2000.0  # 5 NS iterations x 3 GEMMs, scaled to elements
        costs.append((c, n))
    costs.sort(key=lambda t: (-t[0], t[1]))
    load = [0.0] * world
    owner = {}
    for c, n in costs:
        r = min(range(world), key=lambda i: (load[i], i))
        owner[n] = r
        load[r] += c
    return owner


def interleave_by_owner(rows, rank: int, world: int, owner_col: int = 2):
    """Orders push rows round-robin over their destination owners, starting with owner rank + 1: the
    blocks of a push kernel take rows in order, so at any moment each rank writes to every peer and
    every rank receives from all of them (in table order, all ranks would write to the first owner at
    once and leave the other links idle). Rows keep their order within an owner; this rank's own rows
    (local stores) come last in each round."""
    by_owner: dict[int, list] = {}
    for row in rows:
        by_owner.setdefault(int(row[owner_col]), []).append(row)
    order = [(rank + 1 + k) % world for k in range(world)]
    queues = [by_owner.get(o, []) for o in order]
    out = []
    for i in range(max((len(q) for q in queues), default=0)):
        for q in queues:
            if i < len(q):
                out.append(q[i])
    return out


def chunk_ranges(off: int, numel: int, start_in_param: int = 0, size: int = CHUNK):
    out = []
    s = 0
    while s < numel:
        ln = min(size, numel - s)
        out.append((off + s, ln, start_in_param + s))
        s += ln
    return out


class SymmetricBuffer:
    """A device buffer exported over CUDA IPC and opened by every rank of the group."""

    def __init__(self, nbytes: int, group=None):
        self.E = ext()
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.nbytes = nbytes
        self.ptr, handle = self.E.sym_alloc(nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.numpy().tobytes(), group=group)
        self.peer_ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.peer_ptrs.append(self.ptr)
            else:
                self.peer_ptrs.append(self.E.sym_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
        self.device = torch.cuda.current_device()
        self.peers_dev = torch.tensor(self.peer_ptrs, dtype=torch.int64, device="cuda")

    def view(self, numel: int, dtype_code: int, offset_bytes: int = 0) -> torch.Tensor:
        return self.E.sym_view(self.ptr + offset_bytes, numel, dtype_code, self.device)

    def close(self):
        for r, p in enumerate(self.peer_ptrs):
            if r != self.rank:
                try:
                    self.E.sym_close(p)
                except Exception:
                    pass
        self.E.sym_free(self.ptr)


class P2PGradSync:
    """Bucketed, backward-overlapped reduce-scatter + sharded optimizer + parameter gather."""

    def __init__(self, trainer, cfg):
        self.tr = trainer
        self.cfg = cfg
        self.E = ext()
        self.rank, self.world = trainer.rank, trainer.world
        self.wire = WIRE_CODE[cfg.wire_dtype]
        self.budget = float(cfg.comm_timeout_s)
        specs = trainer.model.specs
        self.layout = trainer.layout
        self.ranges = trainer.bucket_ranges
        self.groups = trainer.bucket_groups
        total = trainer.flat_grad.numel()
        self.owner = assign_owners(specs, self.world)
        self.owned_names = {n for n, r in self.owner.items() if r == self.rank}
        dev = trainer.device
        # push reduce-scatter: each owner's parameters get offsets in its owned space; its receive buffer
        # holds one slot of that space per source rank (all slots the same size on every rank)
        owned_tot = [0] * self.world
        self.owned_off = {}
        for n, (off, numel, _) in self.layout.items():
            o = self.owner[n]
            self.owned_off[n] = owned_tot[o]
            owned_tot[o] += -(-numel // ALIGN) * ALIGN
        self.slot_elems = max(max(owned_tot), ALIGN)
        self.recv = SymmetricBuffer(self.world * self.slot_elems * WIRE_BYTES[self.wire])
        self.rflags = SymmetricBuffer(len(self.ranges) * self.world * 8)
        self.recv_peers = torch.tensor(self.recv.peer_ptrs, dtype=torch.int64, device=dev)
        self.rflag_peers = torch.tensor(self.rflags.peer_ptrs, dtype=torch.int64, device=dev)
        self.push_tables, self.own_tables = [], []
        for grp in self.groups:
            rows, mine = [], []
            for n in grp:
                off, numel, _ = self.layout[n]
                for c_off, ln, start in chunk_ranges(off, numel):
                    row = (c_off, ln, self.owner[n], self.owned_off[n] + start)
                    rows.append(row)
                    if self.owner[n] == self.rank:
                        mine.append(row)
            rows = interleave_by_owner(rows, self.rank, self.world)
            self.push_tables.append(torch.tensor(rows, dtype=torch.int64, device=dev).view(-1, 4))
            self.own_tables.append(torch.tensor(mine, dtype=torch.int64, device=dev).view(-1, 4))
        # device skip word (the optimizer kernels read it) and its pinned host copy, read one step late
        # fp16 loss scaling needs the answer on the host, and the top-k path agrees on the host too
        self.device_skip = not trainer.scaler.enabled and not cfg.sparsify.enabled
        self.skip = torch.zeros(1, dtype=torch.int32, device=dev)
        self.snap = torch.zeros(2, dtype=torch.int32).pin_memory()
        self.snap_event = torch.cuda.Event()
        self.snap_pending = False
        self.snap_step, self.snap_names = -1, ()
        # symmetric buffers: params (fp32), flags (int64)
        self.param_buf = SymmetricBuffer(total * 4)
        self.nflags = len(self.ranges) + 2
        self.flags = SymmetricBuffer(self.nflags * 8)
        self.flag_view = self.flags.view(self.nflags, 3)
        self.params_flat = self.param_buf.view(total, 0)
        self.red = torch.zeros(total, dtype=torch.float32, device=dev)
        self.bad = torch.zeros(1, dtype=torch.int32, device=dev)
        # re-point the model parameters into the symmetric parameter buffer
        with torch.no_grad():
            for n, p in trainer.model.named().items():
                off, numel, shape = self.layout[n]
                v = self.params_flat[off:off + numel].view(shape)
                v.copy_(p.data)
                p.data = v
        # the reduced gradients the sharded optimizer consumes (views of ``red``)
        self.red_views = OrderedDict((n, self.red[o:o + k].view(s)) for n, (o, k, s) in self.layout.items())
        self.flag_ptrs = torch.tensor([p for p in self.flags.peer_ptrs], dtype=torch.int64, device=dev)
        # parameter exchange, group by group in forward order: the chunks of each group this rank owns,
        # and one flag slot per (group, source rank) on every rank
        self.fgroups = forward_groups(specs, trainer.model.cfg.n_layer)
        assert sorted(n for g in self.fgroups for n in g) == sorted(self.layout), "forward groups cover every parameter"
        self.push_chunks = []
        for grp in self.fgroups:
            rows = []
            for n in grp:
                if self.owner[n] == self.rank:
                    off, numel, _ = self.layout[n]
                    rows += [(o, ln) for o, ln, _ in chunk_ranges(off, numel)]
            self.push_chunks.append(torch.tensor(sorted(rows), dtype=torch.int64, device=dev).view(-1, 2))
        # the parameters this rank owns, per forward group: with the fused engine the optimizer steps them
        # group by group on the comm stream, each group's push following its update
        self.owned_by_group = [[n for n in grp if n in self.owned_names] for grp in self.fgroups]
        G = len(self.fgroups)
        self.push_flags = SymmetricBuffer(G * self.world * 8)
        self.group_flag_peers = [torch.tensor([p + 8 * g * self.world for p in self.push_flags.peer_ptrs],
                                              dtype=torch.int64, device=dev) for g in range(G)]
        self._build_gather_table(trainer)
        self.group_events = [torch.cuda.Event() for _ in range(G)]
        self.opt_done = torch.cuda.Event()
        self.sparse = cfg.sparsify.enabled
        if self.sparse:
            self._init_sparse(trainer, cfg)
        # high priority: when a compute kernel's CTA retires, the block scheduler hands the SM to a waiting
        # bucket kernel first, so reduces do not queue behind the rest of the backward
        self.comm_stream = torch.cuda.Stream(device=dev, priority=-1)
        self.events = [torch.cuda.Event() for _ in self.ranges]
        self.done = torch.cuda.Event()
        self.epoch = 0
        dist.barrier()

    def _build_gather_table(self, trainer):
        """Per forward group: the segments of parameters other ranks own, with their bf16 shadows."""
        shadows = trainer.engine.shadows if trainer.engine is not None else {}
        self.gather_segs = []
        for grp in self.fgroups:
            rows = []
            for n in grp:
                off, numel, shape = self.layout[n]
                o = self.owner[n]
                if o == self.rank:
                    continue
                sh = shadows.get(n)
                cols = int(shape[-1]) if sh is not None else 0
                ld = int(sh.stride(0)) if sh is not None else 0
                ptr = int(sh.data_ptr()) if sh is not None else 0
                for c_off, ln, start in chunk_ranges(off, numel):
                    rows.append((c_off, ln, o, cols, ld, ptr, start))
            self.gather_segs.append(torch.tensor(rows, dtype=torch.int64, device=trainer.device).view(-1, 7))

    # ------------------------------------------------------------------ top-k + error feedback
    def _init_sparse(self, trainer, cfg):
        """Per (bucket, owner) index/value lists in symmetric memory, sized for the worst case (every
        element kept), so a list can never overflow; error-feedback and velocity buffers are local."""
        sp = cfg.sparsify
        dev = trainer.device
        total = trainer.flat_grad.numel()
        W = self.world
        self.sp_cfg = sp
        self.err = torch.zeros(total, dtype=torch.float32, device=dev)
        self.vel = torch.zeros(total, dtype=torch.float32, device=dev) if sp.momentum_factor > 0 else None
        self.thr = torch.zeros(len(self.ranges), dtype=torch.float32, device=dev)
        # list regions: bucket-major, then owner
        cap = {}
        for b, grp in enumerate(self.groups):
            for o in range(W):
                cap[(b, o)] = sum(self.layout[n][1] for n in grp if self.owner[n] == o)
        base, off = {}, 0
        for b in range(len(self.groups)):
            for o in range(W):
                base[(b, o)] = off
                off += -(-cap[(b, o)] // 8) * 8
        self.list_base = base
        self.sp_idx = SymmetricBuffer(max(off, 8) * 4)
        self.sp_val = SymmetricBuffer(max(off, 8) * 2)
        self.sp_cnt = SymmetricBuffer(len(self.groups) * W * 4 + 16)
        self.sp_cnt_view = self.sp_cnt.view(len(self.groups) * W, 0)  # int32 counters, zeroed per step as fp32 words
        self.sp_peers = torch.tensor([[self.sp_idx.peer_ptrs[r], self.sp_val.peer_ptrs[r], self.sp_cnt.peer_ptrs[r]]
                                      for r in range(W)], dtype=torch.int64, device=dev)
        self.sel_chunks = []
        for b, grp in enumerate(self.groups):
            rows = []
            for n in grp:
                o = self.owner[n]
                noff, numel, _ = self.layout[n]
                for c_off, ln, _ in chunk_ranges(noff, numel, size=1 << 14):
                    rows.append((c_off, ln, base[(b, o)], b * W + o))
            self.sel_chunks.append(torch.tensor(rows, dtype=torch.int64, device=dev).view(-1, 4))
        self.sp_step = 0

    def _sparse_bucket(self, b: int, loss_scale: float) -> None:
        sp = self.sp_cfg
        lo, hi = self.ranges[b]
        mu = sp.momentum_factor
        seed = (self.epoch * 1000003 + b * 7919 + self.rank * 104729) & 0x7FFFFFFF
        self.E.topk_threshold(self.tr.flat_grad, self.err, self.vel, lo, hi, 1.0 / loss_scale, mu, sp.sample_size,
                              sp.top_k_ratio, seed, sp.momentum_masking, self.thr[b:b + 1])
        self.E.topk_select(self.tr.flat_grad, self.err, self.vel, self.sel_chunks[b], 1.0 / loss_scale, mu,
                           sp.momentum_masking, self.thr[b:b + 1], self.sp_idx.ptr, self.sp_val.ptr, self.sp_cnt.ptr)
        self.E.comm_signal(self.flags.ptr + 8 * b, self.epoch + 1)
        self.E.topk_reduce(self.sp_peers, self.flag_ptrs, b, self.epoch + 1, self.list_base[(b, self.rank)],
                           b * self.world + self.rank, self.red, 1.0 / self.world, 32, self.budget)

    # ------------------------------------------------------------------ hooks from the engine
    def bucket_ready(self, b: int, loss_scale: float) -> None:
        """Called on the compute stream when bucket ``b``'s gradients are final for this step."""
        ev = self.events[b]
        ev.record()
        s = self.comm_stream
        s.wait_event(ev)
        lo, hi = self.ranges[b]
        with torch.cuda.stream(s):
            if self.sparse and self.sp_step >= self.sp_cfg.warmup_steps:
                self._sparse_bucket(b, loss_scale)
                return
            ep = self.epoch + 1
            # a small CTA budget: these kernels run beside the backward's compute kernels, and with four
            # vectors in flight per thread 32 CTAs keep about 1 MB of traffic in flight
            self.E.comm_pack_push(self.tr.flat_grad, self.recv_peers, self.rank, self.slot_elems, self.push_tables[b],
                                  self.wire, 1.0 / loss_scale, self.bad, COMM_CTAS)
            self.E.comm_signal_all(self.rflag_peers, self.rank, b, ep, self.bad)
            self.E.comm_reduce_local(self.recv.ptr, self.rflags.ptr, self.world, b, ep, self.slot_elems,
                                     self.own_tables[b], self.red, self.wire, 1.0 / self.world, COMM_CTAS,
                                     self.budget)
            if b == len(self.ranges) - 1:
                self.E.comm_agree(self.rflags.ptr, self.world, b, ep, self.skip, self.budget)

    def begin_step(self) -> None:
        # on the comm stream: the previous step's last bucket kernels there may still read the flag
        with torch.cuda.stream(self.comm_stream):
            self.bad.zero_()
        if self.sparse:
            # the reference counts the step before checking the dense warm-up (gradient-sparsifier.ts:87-91)
            self.sp_step += 1
            if self.sp_step >= self.sp_cfg.warmup_steps:
                self.sp_cnt_view.zero_()
                self.red.zero_()

    # ------------------------------------------------------------------ step
    def step(self, step_idx: int, scale: float, opt) -> bool:
        """The sharded optimizer step and the parameter push, queued without waiting for the device.

        With ``device_skip`` the skip decision is the device word ``agree`` wrote; the host learns it (and
        any status code) from a pinned copy one step later (``poll``), so this returns True before the
        outcome is known. Otherwise (fp16 loss scaling, top-k) the ranks agree on the host first.

        With the fused engine and ``device_skip`` everything after the backward runs on the comm stream and
        the compute stream never waits for it: per forward group, the optimizer steps the parameters this
        rank owns in that group and the exchange pushes them, so the next forward's first layers start
        while the later groups are still being updated. The engine zeroes the gradient buffer only after
        its forward has waited for every group, i.e. after the last bucket kernels of this step read it."""
        timer = self.tr.timer
        epoch = self.epoch + 1
        s = self.comm_stream
        self.poll()
        if self.device_skip and self.tr.engine is not None and self.cfg.overlap_optimizer:
            with torch.cuda.stream(s), traced(timer, "sync.optimizer_exchange"):
                for g in range(len(self.fgroups)):
                    if self.owned_by_group[g]:
                        opt.step({n: self.red_views[n] for n in self.owned_by_group[g]}, skip=self.skip)
                    self._exchange_group(g, epoch)
                self.E.status_snapshot(self.snap, self.skip)
                self.snap_event.record(s)
            self.snap_pending, self.snap_step = True, step_idx
            self.tr.engine.param_ready = self.param_ready
            self.epoch = epoch
            return True
        cur = torch.cuda.current_stream()
        with traced(timer, "sync.comm_tail"):  # the compute stream waits for the last bucket's reduce
            cur.wait_stream(s)
        if self.device_skip:
            ok = True
            with traced(timer, "sync.optimizer"):
                opt.step({n: self.red_views[n] for n in self.owned_names}, skip=self.skip)
            self.E.status_snapshot(self.snap, self.skip)
            self.snap_event.record()
            self.snap_pending, self.snap_step = True, step_idx
        else:
            with traced(timer, "sync.agree"):
                # any non-finite gradient on any rank skips the update everywhere
                flag = self.bad.clone().float()
                dist.all_reduce(flag, op=dist.ReduceOp.MAX)
                status = check_status()
                ok = status == 0 and float(flag.item()) == 0.0
            if status:
                self.tr.log(f"p2p collective timed out (status {status}); step {step_idx} skipped")
            if ok:
                with traced(timer, "sync.optimizer"):
                    opt.step({n: self.red_views[n] for n in self.owned_names})
        self.opt_done.record()
        s.wait_event(self.opt_done)
        with torch.cuda.stream(s), traced(timer, "sync.param_exchange"):
            for g in range(len(self.fgroups)):
                self._exchange_group(g, epoch)
        if self.tr.engine is not None:
            self.tr.engine.param_ready = self.param_ready
        self.epoch = epoch
        return ok

    def _exchange_group(self, g: int, epoch: int) -> None:
        """On the comm stream: push the (possibly unchanged) parameters this rank owns in forward group ``g``
        into every peer's buffer with posted NVLink stores, flag each peer, wait for the other owners'
        flags of the group, refresh the group's bf16 shadows locally and record the group's event; the
        engine's forward waits for that event just before its first kernel that reads group ``g``. Every
        rank's reduce of the last bucket waited for all ranks' last packs, so no peer still reads the
        values being overwritten; pushes only touch a peer's non-owned regions."""
        # COMM_CTAS blocks each: these kernels run beside the forward's, and a refresh block that waits for
        # a flag holds its SM meanwhile
        self.E.comm_push(self.params_flat, self.param_buf.peers_dev, self.rank, self.push_chunks[g], COMM_CTAS)
        self.E.comm_signal_peers(self.group_flag_peers[g], self.rank, epoch)
        self.E.comm_shadow_refresh(self.params_flat, self.push_flags.ptr + 8 * g * self.world, self.world,
                                   self.rank, epoch, self.gather_segs[g], COMM_CTAS, self.budget)
        self.group_events[g].record(self.comm_stream)

    def param_ready(self, g: int) -> None:
        """Makes the current stream wait until forward group ``g`` of the last exchange has arrived."""
        torch.cuda.current_stream().wait_event(self.group_events[g])

    def wait_exchange(self) -> None:
        """Makes the current stream wait for the whole last exchange (before reading every parameter)."""
        torch.cuda.current_stream().wait_event(self.group_events[-1])

    def poll(self, wait: bool = False) -> None:
        """Reads the previous step's device outcome once its copy has landed (or waits for it): a skipped
        step takes back the optimizer's step counters and counts as skipped; a status code is logged and
        cleared."""
        if not self.snap_pending or not (wait or self.snap_event.query()):
            return
        self.snap_event.synchronize()
        self.snap_pending = False
        status, skipped = int(self.snap[0]), int(self.snap[1])
        if skipped:
            self.tr.optimizer.undo_steps(self.owned_names)
            self.tr.skipped += 1
            self.tr.log(f"step {self.snap_step} skipped on the device (non-finite gradient or status {status})")
        if status:
            check_status()  # clears the word for the next steps
            self.tr.log(f"p2p collective reported status {status} at step {self.snap_step}")

    def grad_norm(self) -> float:
        """L2 norm of the step's mean gradient: each rank sums the squares of the reduced gradients it
        owns, one scalar all-reduce adds them up (a collective: every rank calls it on the same steps)."""
        torch.cuda.current_stream().wait_stream(self.comm_stream)  # the reduces may still run there
        sq = torch.zeros((), device=self.red.device)
        for n in self.owned_names:
            sq = sq + self.red_views[n].float().square().sum()
        dist.all_reduce(sq)
        return float(sq.sqrt())

    def close(self):
        torch.cuda.synchronize()
        self.poll(wait=True)
        dist.barrier()
        bufs = [self.recv, self.rflags, self.param_buf, self.flags, self.push_flags]
        if self.sparse:
            bufs += [self.sp_idx, self.sp_val, self.sp_cnt]
        for b in bufs:
            b.close()
