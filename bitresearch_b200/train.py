"""Data-parallel trainer: the fixed-time-budget loop of the reference's ``DistributedTrainer``.

One process per GPU (``torchrun``) or per CPU rank (gloo). Per step (src/distributed/trainer.ts:723-888):

1. next batch (host packer -> pinned buffer -> device);
2. forward + backward: the sm_100a engine (``impl='cuda'``) writes every gradient straight into one
   flat buffer in the reference's variable order; the eager path (``impl='torch'``) uses autograd with
   ``.grad`` views into the same buffer;
3. non-finite check -> skip the update (the reference's overflow/NaN skip, trainer.ts:751-791); with
   ``dtype='fp16'`` the reference's dynamic loss scale is kept (start 1024, halve + skip on
   overflow, double after 2000 good steps);
4. optional top-k + error feedback, then the gradient mean over ranks: in-kernel NVLink
   reduce-scatter (``comm='p2p'``), NCCL all-reduce (``'nccl'``), or the reference's ring over the
   process group (``'ring'``, the CPU/gloo path); an aborted collective skips the update
   (trainer.ts:821-830);
5. schedules (lr multiplier, Muon momentum and weight decay, trainer.ts:577-602) and the optimizer
   (sharded over ranks on the p2p path, followed by the parameter all-gather);
6. metrics: loss, EMA smooth loss (0.9), tokens/s over all ranks, MFU against the measured B200 peak.

``start_training`` stops when ``total_training_time`` (which excludes the first 10 steps,
trainer.ts:986, 1005) reaches ``time_budget`` or at ``max_steps``, then runs ``evaluate_bpb`` on the
held-out split and prints the summary block (trainer.ts:1040-1068) and a ``results.tsv`` row.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time
from collections import OrderedDict

import numpy as np
import torch
import torch.distributed as dist

from . import checkpoint as ckpt
from .config import TrainConfig, apply_overrides, estimate_params, preset
from .data.pipeline import PinnedPrefetcher, make_batch_source
from .data.synthetic import make_token_bytes
from .data.loader import discover_token_bytes, load_token_bytes
from .eval import evaluate_bpb
from .models.gpt import GPT
from .optim.muon_adamw import MuonAdamW, lr_multiplier, muon_momentum, weight_decay_at
from .parallel.comm import flat_layout
from .parallel.ring import RingAllReduce
from .parallel.sparsify import GradientSparsifier
from .utils.timing import traced
from .utils.logging import MetricsLog, ResultsLogger, TrainerMetrics, summary_block

B200_BF16_PEAK_FLOPS = 1630e12  # measured cuBLAS bf16 burst on this hardware (H100: 989.5e12, trainer.ts:102)


class LossScaler:
    """Dynamic loss scale of trainer.ts:159-160, 741-791 (used for fp16 compute)."""

    def __init__(self, enabled: bool, init: float = 1024.0, growth_interval: int = 2000):
        self.enabled = enabled
        self.scale = init if enabled else 1.0
        self.good = 0
        self.growth_interval = growth_interval

    def update(self, overflow: bool) -> None:
        if not self.enabled:
            return
        if overflow:
            self.scale /= 2
            self.good = 0
            return
        self.good += 1
        if self.good >= self.growth_interval:
            self.scale *= 2
            self.good = 0


def init_distributed(backend: str | None = None, timeout_s: float = 120.0):
    """Initialise the default process group from torchrun's env; returns (rank, world, local_rank)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s),
                                **({"device_id": torch.device("cuda", local)} if backend == "nccl" else {}))
    return rank, world, local


class Trainer:
    def __init__(self, cfg: TrainConfig, device: str | torch.device | None = None, log=None):
        self.cfg = cfg
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        if cfg.elastic_join and not dist.is_initialized():
            # a process joining a running elastic job: its launcher's RANK / WORLD_SIZE size the batch
            self.rank = int(os.environ.get("RANK", "0"))
            self.world = int(os.environ.get("WORLD_SIZE", "1"))
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        self.is_cuda = self.device.type == "cuda"
        self._log = log or (lambda m: print(m, flush=True) if self.rank == 0 else None)
        self.metrics = TrainerMetrics()
        self.total_training_time = 0.0
        self.start_time = 0.0
        self.status_server = None
        self.membership = None
        self.timer = None  # PhaseTimer when trace_phases is on
        self.phase_ms: dict[str, float] = {}
        self._profiler = None
        self.egroup = None  # ElasticGroup of the current ring (elastic ring path)
        self._comm_failed = False
        self.running = False
        self.scaler = LossScaler(cfg.dtype == "fp16")
        self.skipped = 0
        self.model: GPT | None = None
        self.engine = None
        self.optimizer: MuonAdamW | None = None
        self.comm = None
        self.sparsifier: GradientSparsifier | None = None
        self.prefetch = None

    def log(self, msg: str) -> None:
        self._log(msg)

    # ------------------------------------------------------------------ setup
    def initialize(self) -> None:
        cfg = self.cfg
        torch.manual_seed(cfg.seed)
        self.model = GPT(cfg.model, init="karpathy", seed=42, device=self.device)
        self._fwd = self.model.forward_torch
        if cfg.torch_compile and cfg.impl == "torch" and self.is_cuda:
            self.model.attn_impl = "flex"
            self._fwd = torch.compile(self.model.forward_torch)
        self.specs = self.model.specs
        self.metrics.num_params_m = self.model.num_params() / 1e6
        self.flops_per_token = self.model.estimate_flops_per_token()
        if self.rank == 0:
            self.log(f"model: {self.metrics.num_params_m:.1f}M params (estimate {estimate_params(cfg.model) / 1e6:.2f}M), "
                     f"{self.flops_per_token / 1e6:.1f} MFLOP/token, world={self.world}, impl={cfg.impl}")
        T = cfg.model.sequence_len
        per_rank_tokens = cfg.total_batch_tokens // self.world
        if per_rank_tokens % T:
            raise ValueError("total_batch_tokens / world must be a multiple of sequence_len")
        rows = per_rank_tokens // T
        self.device_batch = min(cfg.device_batch, rows)
        if rows % self.device_batch:
            raise ValueError(f"per-rank rows {rows} not divisible by device_batch {self.device_batch}")
        self.grad_accum = rows // self.device_batch
        # one flat fp32 gradient buffer ordered by backward completion (one contiguous range per
        # communication bucket), with a view per parameter
        self.layout, self.bucket_ranges, self.bucket_groups, total = flat_layout(self.specs, cfg.model.n_layer)
        self.flat_grad = torch.zeros(total, dtype=torch.float32, device=self.device)
        self.grad_views: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        for name, _, _ in self.specs:
            off, numel, shape = self.layout[name]
            self.grad_views[name] = self.flat_grad[off:off + numel].view(shape)
        owned = None
        if cfg.impl == "cuda":
            from .models.engine import FusedGPTEngine
            self.engine = FusedGPTEngine(self.model, self.grad_views, self.device_batch, T, flat_grad=self.flat_grad)
            if self.world > 1 and cfg.comm == "p2p":
                from .parallel.comm import P2PGradSync
                self.comm = P2PGradSync(self, cfg)
                owned = self.comm.owned_names
                self.engine.bucket_hook = self.comm.bucket_ready
        else:
            for name, p in self.model.named().items():
                p.grad = self.grad_views[name]
        if (self.world > 1 or cfg.elastic_join) and cfg.comm == "ring":
            if cfg.elastic or cfg.elastic_join:
                self._init_elastic()
            self.comm = RingAllReduce(wire_dtype=cfg.wire_dtype, timeout_s=self._ring_timeout(), log=self.log,
                                      elastic=self.egroup)
        fused_comm = cfg.impl == "cuda" and cfg.comm == "p2p" and self.world > 1
        if cfg.sparsify.enabled and not fused_comm:
            self.sparsifier = GradientSparsifier(cfg.sparsify.top_k_ratio, cfg.sparsify.warmup_steps,
                                                 cfg.sparsify.sample_size, cfg.sparsify.momentum_factor,
                                                 seed=cfg.seed + self.rank,
                                                 momentum_masking=cfg.sparsify.momentum_masking)
        self.optimizer = MuonAdamW(
            self.model.named(), self.model.param_groups(), model_dim=cfg.model.n_embd,
            unembedding_lr=cfg.unembedding_lr, embedding_lr=cfg.embedding_lr, matrix_lr=cfg.matrix_lr,
            scalar_lr=cfg.scalar_lr, weight_decay=cfg.weight_decay, adam_betas=cfg.adam_betas, ns_steps=cfg.ns_steps,
            beta2=cfg.muon_beta2, ns_dtype=cfg.ns_dtype if self.is_cuda else "fp32", owned=owned,
            impl="cuda" if cfg.impl == "cuda" else "torch",
            shadows=self.engine.shadows if self.engine is not None else None)
        if self.engine is not None:
            self.engine.attach_optimizer(self.optimizer)
        if cfg.trace_phases and self.is_cuda:
            from .utils.timing import PhaseTimer
            self.timer = PhaseTimer()
            if self.engine is not None:
                self.engine.timer = self.timer
        # data
        self.train_source = make_batch_source(cfg, "train", self.rank, self.world)
        if cfg.data in ("tokens", "documents"):
            # explicit table, else the one the manifest / data directory provides, else all ones (the
            # reference's avgBytesPerToken = 1 fallback)
            tb_path = cfg.token_bytes_path or discover_token_bytes(cfg.data_path)
            self.token_bytes = load_token_bytes(tb_path, cfg.model.vocab_size)
        else:
            self.token_bytes = make_token_bytes(cfg.model.vocab_size, cfg.token_bytes_max)
        if self.is_cuda:
            self.prefetch = PinnedPrefetcher(self.train_source, self.device_batch, T, self.device)
        if getattr(self, "_join_resync", False):  # a joining process takes the ring's state
            self._join_resync = False
            self._resync(member=False)
            self.log(f"joined the ring at step {self.metrics.step}: {self.egroup.ring.peers}")

    # ------------------------------------------------------------------ batches
    def next_batch(self):
        if self.prefetch is not None:
            return self.prefetch.get()
        x, y = self.train_source.next(self.device_batch, self.cfg.model.sequence_len)
        return (torch.as_tensor(np.ascontiguousarray(x), device=self.device),
                torch.as_tensor(np.ascontiguousarray(y), device=self.device))

    # ------------------------------------------------------------------ step
    def _forward_backward(self, x, y, scale: float):
        if self.engine is not None:
            return self.engine.forward_backward(x, y, loss_scale=scale / self.grad_accum,
                                                accumulate=self._micro > 0,
                                                last_micro=self._micro == self.grad_accum - 1, grad_scale=scale)
        cd = torch.bfloat16 if self.is_cuda and self.cfg.dtype == "bf16" else (
            torch.float16 if self.is_cuda and self.cfg.dtype == "fp16" else None)
        loss = self._fwd(x, y, compute_dtype=cd, exact_ce=not self.is_cuda)
        (loss * (scale / self.grad_accum)).backward()
        return loss.detach()

    def train_step(self, batch=None, sync: bool = True):
        """One optimizer step over ``grad_accum`` micro-batches.

        ``batch``: None (draw from the data pipeline), one ``(inputs, targets)`` pair used for every
        micro-batch, or a list with one pair per micro-batch. Returns the host loss, or the device
        loss tensor with ``sync=False`` (no device->host read).
        """
        cfg = self.cfg
        t0 = time.perf_counter()
        progress = min(self.total_training_time / cfg.time_budget, 1.0)
        if self.engine is None:
            self.flat_grad.zero_()
        losses = []
        scale = self.scaler.scale
        if self.comm is not None and hasattr(self.comm, "begin_step"):
            self.comm.begin_step()
        for self._micro in range(self.grad_accum):
            with traced(self.timer, "data"):
                if batch is None:
                    x, y = self.next_batch()
                elif isinstance(batch, list):
                    x, y = batch[self._micro]
                else:
                    x, y = batch
            if self.engine is None:
                with traced(self.timer, "forward_backward"):
                    losses.append(self._forward_backward(x, y, scale))
            else:
                losses.append(self._forward_backward(x, y, scale))
        loss_t = losses[0].float() if len(losses) == 1 else torch.stack(losses).float().mean()
        t_compute = time.perf_counter()
        with traced(self.timer, "sync_update"):  # gradient sync tail, optimizer, parameter exchange
            ok = self._sync_and_update(progress, scale)
        if not sync:
            self.metrics.step += 1
            return loss_t
        loss = float(loss_t)  # device -> host read of the step result
        if self.timer is not None:
            self.phase_ms = self.timer.collect()
        if self.engine is not None:
            st = self.engine.status()
            if st:
                raise RuntimeError(f"a kernel gave up a bounded wait (status {st}) at step {self.metrics.step}")
        if not math.isfinite(loss):
            self.log(f"non-finite loss at step {self.metrics.step}")
        self._update_metrics(loss, t0, t_compute, ok)
        return loss

    def _sync_and_update(self, progress: float, scale: float) -> bool:
        cfg = self.cfg
        log_step = bool(cfg.log_every) and self.metrics.step % cfg.log_every == 0
        if self.comm is not None and hasattr(self.comm, "step"):  # in-kernel p2p path
            ok = self.comm.step(self.metrics.step, scale, self._set_schedules(progress))
            if log_step:
                self.metrics.grad_norm = self.comm.grad_norm()
            return ok
        g = self.flat_grad
        finite = torch.isfinite(g).all()
        if scale != 1.0:
            g.div_(scale)
        overflow = not bool(finite)
        if self.scaler.enabled and not overflow:
            overflow = float(g.abs().max()) * scale > 65000
        if self.world > 1:
            flag = torch.tensor([1.0 if overflow else 0.0], device=self.device)
            if isinstance(self.comm, RingAllReduce):
                flag = flag.cpu()
            if not self._group_all_reduce(flag, dist.ReduceOp.MAX):
                self.log(f"peer lost at step {self.metrics.step}, skipping optimizer update")
                self.skipped += 1
                return False
            overflow = bool(flag.item() > 0)
        self.scaler.update(overflow)
        if overflow:
            self.skipped += 1
            return False
        if self.sparsifier is not None:
            sp = self.sparsifier.sparsify(g)
            if self.metrics.step % 50 == 0:
                self.log(f"sparsification: {sp.indices.numel()}/{sp.length} kept "
                         f"({100 * GradientSparsifier.compression_ratio(sp):.1f}% of dense)")
        t_ar = time.perf_counter()
        if self.world > 1:
            if isinstance(self.comm, RingAllReduce):
                red = self.comm.all_reduce(g, self.metrics.step)
                if red is None:
                    self.log(f"all-reduce aborted at step {self.metrics.step}, skipping optimizer update")
                    self.skipped += 1
                    self._comm_failed = self.egroup is not None
                    return False
                g.copy_(red)
            else:
                dist.all_reduce(g, op=dist.ReduceOp.AVG if self.is_cuda else dist.ReduceOp.SUM)
                if not self.is_cuda:
                    g.div_(self.world)
        if self.is_cuda:
            torch.cuda.synchronize(self.device) if cfg.log_every and self.metrics.step % cfg.log_every == 0 else None
        self.metrics.all_reduce_time_ms = (time.perf_counter() - t_ar) * 1e3
        if log_step:  # the mean gradient's L2 norm (logging steps only: it reads back one scalar)
            self.metrics.grad_norm = float(g.norm())
        self._set_schedules(progress)
        self.optimizer.step(self.grad_views)
        return True

    def _set_schedules(self, progress: float):
        cfg = self.cfg
        o = self.optimizer
        o.lr_multiplier = lr_multiplier(progress, cfg.warmup_ratio, cfg.warmdown_ratio, cfg.final_lr_frac)
        o.muon_momentum = muon_momentum(self.metrics.step)
        o.muon_weight_decay = weight_decay_at(progress, cfg.weight_decay)
        return o

    def _update_metrics(self, loss: float, t0: float, t_compute: float, ok: bool):
        m = self.metrics
        tokens = self.device_batch * self.grad_accum * self.cfg.model.sequence_len * self.world
        m.step += 1
        m.loss = loss
        m.smooth_loss = loss if m.smooth_loss == 0 else 0.9 * m.smooth_loss + 0.1 * loss
        m.total_tokens += tokens
        m.compute_time_ms = (t_compute - t0) * 1e3
        m.step_time_ms = (time.perf_counter() - t0) * 1e3
        m.tokens_per_sec = tokens / max(m.step_time_ms / 1e3, 1e-9)
        m.elapsed_seconds = time.perf_counter() - self.start_time if self.start_time else 0.0
        m.peers_connected = self.world
        m.skipped_steps = self.skipped
        steady = max(1, m.step - self.cfg.warmup_steps_excluded)
        if self.total_training_time > 0:
            m.mfu_percent = 100 * self.flops_per_token * tokens * steady / self.total_training_time / (
                B200_BF16_PEAK_FLOPS * self.world)

    # ------------------------------------------------------------------ eval
    def per_token_nats(self, x, y):
        if self.engine is not None:
            return self.engine.per_token_nats(x, y)
        cd = torch.bfloat16 if self.is_cuda else None
        with torch.no_grad():
            return self.model.forward_torch(x, y, reduction="none", compute_dtype=cd, exact_ce=True)

    def evaluate_bpb(self, batch: int | None = None) -> float:
        cfg = self.cfg
        B = batch or self.device_batch
        val = make_batch_source(cfg, "val", 0, 1)
        # ranks split the eval batches; sums are reduced over the group
        tokens = max(cfg.eval_tokens // self.world, B * cfg.model.sequence_len)
        bpb, nats, nbytes = evaluate_bpb(self.per_token_nats, _Skip(val, self.rank, self.world, B, cfg.model.sequence_len),
                                         self.token_bytes, B, cfg.model.sequence_len, tokens, self.device)
        if self.world > 1:
            t = torch.tensor([nats, nbytes], dtype=torch.float64,
                             device=self.device if self.is_cuda and self.egroup is None else "cpu")
            if self._group_all_reduce(t, dist.ReduceOp.SUM):
                nats, nbytes = float(t[0]), float(t[1])
            else:
                self.log("evaluation sums could not be reduced (peer lost); val_bpb is this rank's share")
            bpb = nats / (math.log(2) * nbytes) if nbytes > 0 else 0.0
        self.metrics.val_bpb = bpb
        if cfg.data == "markov" and self.rank == 0 and "val_bpb_floor" not in self.metrics.extra:
            from .data.pipeline import markov_floor
            fb, fn = markov_floor(cfg, self.token_bytes, min(cfg.eval_tokens, 1 << 22), B)
            self.metrics.extra.update(val_bpb_floor=fb, val_nats_floor=fn)
        return bpb

    # ------------------------------------------------------------------ loop
    def _profile_tick(self) -> None:
        """torch.profiler over steps [a, b) of ``profile_steps="a:b"``; writes a Chrome trace per rank.
        Timings read under the profiler are not benchmark numbers."""
        spec = self.cfg.profile_steps
        if not spec:
            return
        a, b = (int(v) for v in spec.split(":"))
        step = self.metrics.step
        if step == a and self._profiler is None:
            acts = [torch.profiler.ProfilerActivity.CPU] + (
                [torch.profiler.ProfilerActivity.CUDA] if self.is_cuda else [])
            self._profiler = torch.profiler.profile(activities=acts, record_shapes=False, acc_events=True)
            self._profiler.__enter__()
        elif step == b and self._profiler is not None:
            self._profiler.__exit__(None, None, None)
            os.makedirs(self.cfg.profile_dir, exist_ok=True)
            path = os.path.join(self.cfg.profile_dir, f"trace_rank{self.rank}_steps{a}-{b}.json")
            self._profiler.export_chrome_trace(path)
            self._profiler = None
            self.log(f"profiler trace: {path}")

    def _group_all_reduce(self, t: torch.Tensor, op) -> bool:
        """All-reduce over the current group (the elastic ring's gloo group, else the default group);
        False when a member of the elastic ring is gone."""
        if self.egroup is not None:
            ok = self.egroup.all_reduce(t, op)
            self._comm_failed |= not ok
            return ok
        dist.all_reduce(t, op=op)
        return True

    def _agreed_time(self, local_s: float) -> float:
        """The slowest rank's training time, so every rank stops on the same step and follows the
        same learning-rate schedule. Each browser peer of the reference keeps its own clock
        (src/distributed/trainer.ts:986-1005) and its ring tolerates a peer that stops early; here the
        ranks' collectives must stay matched, so the stop decision is collective."""
        nccl = self.egroup is None and self.is_cuda and dist.get_backend() == "nccl"
        t = torch.tensor([local_s], dtype=torch.float64, device=self.device if nccl else torch.device("cpu"))
        if not self._group_all_reduce(t, dist.ReduceOp.MAX):
            return local_s
        return float(t.item())

    # ------------------------------------------------------------------ elastic ring
    def _init_elastic(self) -> None:
        """Registers this rank in the job store's membership room, starts its heartbeat and builds the
        first ring's gloo group (the reference's ring formation, server/signaling.ts:75-119). With
        ``elastic_join`` the process instead waits until the running ring takes it in (the server
        re-forms the ring on join, server/signaling.ts:210-213); it receives the state once the
        optimizer exists (end of ``initialize``)."""
        from .parallel.membership import ElasticGroup, Membership, store_client
        cfg = self.cfg
        self._store = store_client()
        # a joining process gets an id of its own, so a restarted rank never collides with its old entry
        pid = f"rank{self.rank:05d}" + (f"-join{os.getpid()}" if cfg.elastic_join else "")
        self.membership = Membership(self._store, pid, room="train", heartbeat_s=cfg.heartbeat_s,
                                     dead_after_s=cfg.dead_after_s, heartbeat_store=store_client())
        self._ring_seq = self.membership.latest_published()
        self.membership.register()
        self.membership.start()
        if cfg.elastic_join:
            self.log(f"{pid} waiting to be taken into the ring")
            self._ring_seq, ring = self.membership.wait_published(self._ring_seq, cfg.reform_timeout_s)
            self._join_resync = True
        else:
            ring = self.membership.wait_for(self.world, cfg.reform_timeout_s)
        self.egroup = ElasticGroup(self._store, ring, room="train", timeout_s=self._ring_timeout())
        self.rank, self.world = ring.position, ring.total

    def _ring_timeout(self) -> float:
        """``comm_timeout_s``, or with 0 the membership's dynamic timeout max(10, 3 * rtt + 5) s, read at ring
        formation as the reference does (webrtc-mesh.ts:99-109, trainer.ts:656-659)."""
        if self.cfg.comm_timeout_s > 0 or self.membership is None:
            return self.cfg.comm_timeout_s if self.cfg.comm_timeout_s > 0 else 10.0
        return self.membership.dynamic_timeout_s

    def _reform(self) -> None:
        """After a step that lost a peer: wait until membership drops it, form the new ring with its own
        gloo group and re-sync the state from a surviving member. The reference re-forms on the server's
        ``peer-left`` (server/signaling.ts:264-295, trainer.ts:654-668); its ranks may keep different
        weights when some completed the aborted step, which the re-sync removes.

        The first surviving member decides the new ring (survivors plus any peers that joined the room)
        and publishes it; every member, and every joining process, forms its ring from that list, so
        all of them build the same group whatever heartbeats each of them saw. While fewer than
        ``min_ring_size`` peers are alive the ring pauses, as the reference does with minRingSize
        (src/distributed/trainer.ts:992-999), and stops after ``reform_timeout_s``."""
        cfg = self.cfg
        old = self.egroup.ring.peers
        me = self.membership.peer_id
        self.log(f"peer lost at step {self.metrics.step}; re-forming the ring of {len(old)}")
        changed = self.membership.wait_for_change(old, cfg.reform_timeout_s)
        surv = sorted(set(changed.peers) & set(old))
        small = len(surv) < cfg.min_ring_size
        if small:
            self.log(f"ring too small ({len(surv)}/{cfg.min_ring_size}), waiting up to {cfg.reform_timeout_s:.0f} s")
        try:
            if surv and surv[0] == me:
                deadline = time.time() + cfg.reform_timeout_s
                while len(alive := self.membership.alive_peers()) < cfg.min_ring_size:
                    if time.time() > deadline:
                        raise TimeoutError(f"only {len(alive)} peers alive")
                    time.sleep(min(0.05, cfg.heartbeat_s))
                self.membership.publish_ring(sorted((set(alive) - set(old)) | set(surv)))
            self._ring_seq, ring = self.membership.wait_published(self._ring_seq, cfg.reform_timeout_s)
        except TimeoutError as e:
            if small:
                raise RuntimeError(f"ring stayed below min_ring_size={cfg.min_ring_size}: {e}") from e
            raise RuntimeError(f"ring re-formation failed: {e}") from e
        self._switch_ring(ring, survivors=old)

    def _take_in_joiners(self) -> None:
        """Every ``join_check_steps`` steps: the ring's first member looks for peers that joined the room;
        if there are any, all members agree (one all-reduce), it publishes the larger ring and everyone,
        the newcomers included, switches to it and re-syncs the state."""
        cfg = self.cfg
        ring = self.egroup.ring
        new = []
        if ring.position == 0:
            new = sorted(set(self.membership.alive_peers()) - set(ring.peers))
        flag = torch.tensor([1.0 if new else 0.0])
        if not self._group_all_reduce(flag, dist.ReduceOp.MAX) or flag.item() == 0:
            return
        if ring.position == 0:
            self.log(f"taking in {new} at step {self.metrics.step}")
            self.membership.publish_ring(sorted(set(ring.peers) | set(new)))
        self._ring_seq, nring = self.membership.wait_published(self._ring_seq, cfg.reform_timeout_s)
        self._switch_ring(nring, survivors=ring.peers)

    def _switch_ring(self, ring, survivors: list[str]) -> None:
        """Builds ``ring``'s gloo group and ring all-reduce, then re-syncs the state from the first
        member that was already training (never from a process that just joined)."""
        from .parallel.membership import ElasticGroup
        cfg = self.cfg
        self.egroup = ElasticGroup(self._store, ring, room="train", timeout_s=self._ring_timeout())
        self.comm = RingAllReduce(wire_dtype=cfg.wire_dtype, timeout_s=self._ring_timeout(), log=self.log,
                                  elastic=self.egroup)
        self.rank, self.world = ring.position, ring.total
        self._resync(member=self.membership.peer_id in survivors)
        self._comm_failed = False
        self.log(f"ring re-formed: version {ring.version}, {ring.total} peers {ring.peers}")

    def _resync(self, member: bool = True) -> None:
        """Broadcasts weights, optimizer state, loss scale and schedule state from the lowest ring position
        held by a member that was training before (``member``); a process that just joined receives."""
        g = self.egroup
        pos = torch.tensor([float(g.rank if member else g.size)])
        if not g.all_reduce(pos, dist.ReduceOp.MIN) or int(pos.item()) >= g.size:
            raise RuntimeError("state re-sync failed (no member holds the training state)")
        root = int(pos.item())
        if g.rank == root:
            tensors, meta = self.checkpoint_state()
            buf = ckpt.to_bytes(tensors, meta)
            n = torch.tensor([len(buf)], dtype=torch.int64)
        else:
            n = torch.zeros(1, dtype=torch.int64)
        if not g.broadcast(n, root):
            raise RuntimeError("state re-sync failed (size)")
        data = (torch.frombuffer(bytearray(buf), dtype=torch.uint8) if g.rank == root
                else torch.empty(int(n.item()), dtype=torch.uint8))
        if not g.broadcast(data, root):
            raise RuntimeError("state re-sync failed (payload)")
        if g.rank != root:
            tensors, meta = ckpt.from_bytes(data.numpy().tobytes())
            info = ckpt.restore(self.model, tensors, meta, self.optimizer, log=self.log)
            self.scaler.scale = float(info.get("lossScale", self.scaler.scale) or self.scaler.scale)
            self.metrics.step = int(info.get("step", self.metrics.step) or 0)
            self.metrics.total_tokens = int(info.get("totalTokens", self.metrics.total_tokens) or 0)
            self.total_training_time = float(info.get("totalTrainingTime", self.total_training_time) or 0.0)
            self.metrics.smooth_loss = float(info.get("smoothLoss", self.metrics.smooth_loss) or 0.0)
            if self.engine is not None:
                self.engine.refresh_shadows()

    def start_training(self) -> TrainerMetrics:
        cfg = self.cfg
        if self.model is None:
            self.initialize()
        self.running = True
        self.start_time = time.perf_counter()
        if cfg.status_port >= 0 and self.rank == 0 and self.status_server is None:
            from .utils.status import StatusServer
            self.status_server = StatusServer(self.status, lambda: self.metrics.to_dict(), port=cfg.status_port)
            self.status_server.start()
            self.log(f"status: {self.status_server.url}/status and /metrics")
        jl = MetricsLog(cfg.metrics_jsonl if self.rank == 0 else "")
        while self.running and self.metrics.step < cfg.max_steps:
            if self.metrics.step > cfg.warmup_steps_excluded and self.total_training_time >= cfg.time_budget:
                self.log("time budget exhausted")
                break
            t0 = time.perf_counter()
            loss = self.train_step()
            dt = time.perf_counter() - t0
            if self.metrics.step > cfg.warmup_steps_excluded:
                self.total_training_time += dt
            if self.world > 1 and not self._comm_failed:
                self.total_training_time = self._agreed_time(self.total_training_time)
            if self._comm_failed and self.egroup is not None:
                self._reform()
            elif (self.egroup is not None and cfg.join_check_steps > 0
                  and self.metrics.step % cfg.join_check_steps == 0):
                self._take_in_joiners()
                if self._comm_failed:
                    self._reform()
            m = self.metrics
            if cfg.log_every and m.step % cfg.log_every == 0:
                lrm = lr_multiplier(min(self.total_training_time / cfg.time_budget, 1), cfg.warmup_ratio,
                                    cfg.warmdown_ratio, cfg.final_lr_frac)
                self.log(f"Step {m.step} | loss={loss:.6f} | smooth={m.smooth_loss:.6f} | grad={m.grad_norm:.4f} | "
                         f"lrm={lrm:.2f} | {m.tokens_per_sec:.0f} tok/s | peers={m.peers_connected} | "
                         f"{m.elapsed_seconds:.0f}s")
            rec = {"step": m.step, "loss": loss, "smooth_loss": m.smooth_loss, "tokens_per_sec": m.tokens_per_sec,
                   "step_ms": m.step_time_ms, "all_reduce_ms": m.all_reduce_time_ms, "mfu": m.mfu_percent}
            if self.phase_ms:
                rec["phases_ms"] = self.phase_ms
                if cfg.log_every and m.step % cfg.log_every == 0:
                    self.log("phases: " + " | ".join(f"{k} {v:.2f} ms" for k, v in self.phase_ms.items()))
            if self.status_server is not None and cfg.log_every and m.step % cfg.log_every == 0:
                self.status_server.publish({"type": "metrics", **rec, "grad_norm": m.grad_norm})
            jl.write(rec)
            self._profile_tick()
            if cfg.checkpoint_interval > 0 and m.step % cfg.checkpoint_interval == 0:
                self.save_checkpoint()
        self.log("running final BPB evaluation")
        self.evaluate_bpb()
        total = time.perf_counter() - self.start_time
        peak = torch.cuda.max_memory_allocated(self.device) / 2 ** 20 if self.is_cuda else 0.0
        if self.status_server is not None:
            self.status_server.publish({"type": "training-complete", "val_bpb": self.metrics.val_bpb,
                                        "num_steps": self.metrics.step, "training_seconds": self.total_training_time,
                                        "total_seconds": total, **self.metrics.extra})
        if self.rank == 0:
            print(summary_block(self.metrics, self.total_training_time, total, peak, cfg.model.n_layer), flush=True)
            if cfg.results_tsv:
                ResultsLogger(cfg.results_tsv).log(
                    self.metrics.val_bpb, peak, "keep" if self.metrics.val_bpb > 0 else "crash",
                    f"step {self.metrics.step} | {self.metrics.num_params_m:.1f}M params | depth={cfg.model.n_layer}")
        return self.metrics

    def status(self) -> dict:
        """The reference's signalling-server status fields (one room, one compute peer per rank, a static
        ring) with this job's metrics under ``training``."""
        joined = getattr(self, "_joined_ms", None) or time.time() * 1e3
        self._joined_ms = joined
        peers = [{"id": f"rank{r}", "room": "default", "position": r, "peerType": "compute", "joinedAt": joined}
                 for r in range(self.world)]
        m = self.metrics.to_dict()
        m.update(time_budget=self.cfg.time_budget, training_seconds=self.total_training_time,
                 running=self.running)
        return {"rooms": ["default"], "peers": peers, "ringVersion": 1, "totalPeers": self.world,
                "computePeers": self.world, "observerPeers": 0, "swarms": {}, "training": m}

    def stop(self) -> None:
        self.running = False

    def destroy(self) -> None:
        self.stop()
        if self.membership is not None:
            self.membership.leave()
            self.membership = None
        if self.status_server is not None:
            self.status_server.stop()
            self.status_server = None
        if self.prefetch is not None:
            self.prefetch.close()
        if self.comm is not None and hasattr(self.comm, "close"):
            self.comm.close()

    # ------------------------------------------------------------------ checkpoints
    def join_streams(self) -> None:
        """Makes the current stream wait for the work this trainer queued on side streams (the data-parallel
        parameter exchange that overlaps the next forward): an event recorded after this call covers every
        step so far."""
        if self.comm is not None and hasattr(self.comm, "comm_stream"):
            torch.cuda.current_stream().wait_stream(self.comm.comm_stream)

    def checkpoint_state(self):
        self.join_streams() if self.is_cuda else None
        if self.engine is not None:
            self.engine.sync_params_to_model()
        return ckpt.build_state(
            self.model, self.optimizer, step=self.metrics.step, loss_scale=self.scaler.scale,
            total_tokens=self.metrics.total_tokens,
            extra_meta={"totalTrainingTime": self.total_training_time, "smoothLoss": self.metrics.smooth_loss,
                        "trainConfig": self.cfg.to_json()})

    def save_checkpoint(self, path: str | None = None) -> str:
        tensors, meta = self.checkpoint_state()
        if self.world > 1:
            # each rank holds the optimizer state of its own shard; weights are replicated
            own = set(self.optimizer.state)
            t_local = OrderedDict((k, v) for k, v in tensors.items()
                                  if not (k.startswith("adam_") or k.startswith("muon_")) or
                                  k.split("_", 2)[-1] in own)
            d = path or os.path.join(self.cfg.checkpoint_dir, f"step{self.metrics.step:06d}")
            ckpt.save_sharded(d, self.rank, self.world, t_local if self.rank == 0 else
                              OrderedDict((k, v) for k, v in t_local.items() if k.startswith(("adam_", "muon_"))), meta)
            # every shard is on disk before position 0 merges (a blocking gloo all-reduce over the live ring
            # in elastic mode, where the default group may contain a lost rank)
            if self.egroup is None:
                dist.barrier()
            elif not self.egroup.all_reduce(torch.zeros(1), dist.ReduceOp.SUM):
                raise RuntimeError("a peer was lost while saving a checkpoint")
            if self.rank == 0:
                out = d + ".safetensors"
                ckpt.merge_shards(d, out, order=[n for n, _, _ in self.specs])
                return out
            return d
        path = path or os.path.join(self.cfg.checkpoint_dir, ckpt.checkpoint_filename(self.metrics.step))
        ckpt.save(path, tensors, meta)
        self.log(f"checkpoint saved: {path}")
        return path

    def load_checkpoint(self, path: str) -> dict:
        if self.model is None:
            raise RuntimeError("Cannot load checkpoint: model not initialized. Call initialize() first.")
        tensors, meta = ckpt.load(path)
        info = ckpt.restore(self.model, tensors, meta, self.optimizer, log=self.log)
        self.metrics.step = int(info.get("step", 0) or 0)
        self.scaler.scale = float(info.get("lossScale", 1.0) or 1.0)
        self.metrics.total_tokens = int(info.get("totalTokens", 0) or 0)
        self.total_training_time = float(info.get("totalTrainingTime", 0.0) or 0.0)
        self.metrics.smooth_loss = float(info.get("smoothLoss", 0.0) or 0.0)
        if self.engine is not None:
            self.engine.refresh_shadows()
        self.log(f"resumed from step {self.metrics.step} ({info['restored']} weights)")
        return info


class _Skip:
    """Round-robin view of a batch source: rank r takes batches r, r+W, r+2W, ..."""

    def __init__(self, src, rank, world, B, T):
        self.src, self.rank, self.world, self.B, self.T = src, rank, world, B, T
        self.first = True

    def next(self, B, T):
        skip = self.rank if self.first else self.world - 1
        self.first = False
        for _ in range(skip):
            self.src.next(B, T)
        return self.src.next(B, T)


def _launch_peers(n: int, argv: list[str]) -> int:
    """Re-runs this CLI as ``n`` local ranks through torch.distributed.run on 127.0.0.1 (the reference's
    launcher opens N browser tabs, scripts/launch.ts:83-182)."""
    import socket
    import subprocess
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={port}", "-m", "bitresearch_b200.train", *argv]
    return subprocess.call(cmd)


def main(argv=None):
    ap = argparse.ArgumentParser(description="bitresearch-b200 data-parallel GPT trainer")
    ap.add_argument("--preset", default=None, help="default d512; with --resume, the checkpoint's own config")
    ap.add_argument("--resume", default="")
    # the reference launcher's flags (scripts/launch.ts:13-23); the same settings as key=value work too
    ap.add_argument("--peers", type=int, default=0, help="launch N local ranks (one per GPU) and train on all")
    ap.add_argument("--max-steps", type=int, default=0)
    ap.add_argument("--max-seconds", "--timeout", dest="max_seconds", type=float, default=0.0,
                    help="training time budget in seconds")
    ap.add_argument("overrides", nargs="*", help="key=value config overrides (e.g. max_steps=100 model.n_layer=4)")
    raw = list(sys.argv[1:] if argv is None else argv)
    args = ap.parse_args(raw)
    if args.peers > 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        rest, skip = [], False
        for a in raw:  # drop --peers N / --peers=N, keep everything else for the ranks
            if skip:
                skip = False
                continue
            if a == "--peers":
                skip = True
                continue
            if not a.startswith("--peers="):
                rest.append(a)
        return _launch_peers(args.peers, rest)
    extra = ([f"max_steps={args.max_steps}"] if args.max_steps else []) + (
        [f"time_budget={args.max_seconds}"] if args.max_seconds else [])
    if args.resume and args.preset is None:  # continue with the configuration the checkpoint was trained with
        from .eval import _config_from_checkpoint
        base = _config_from_checkpoint(args.resume, preset("d512"))
    else:
        base = preset(args.preset or "d512")
    cfg = apply_overrides(base, list(args.overrides) + extra)
    rank, world, local = init_distributed("nccl" if torch.cuda.is_available() and cfg.impl != "cpu" else "gloo")
    if not torch.cuda.is_available():
        cfg.impl = "torch"
    tr = Trainer(cfg)
    tr.initialize()
    if args.resume:
        tr.load_checkpoint(args.resume)
    try:
        tr.start_training()
    finally:
        tr.destroy()
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
