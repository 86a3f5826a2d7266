"""Training-throughput benchmark: the d512 depth-8 autoresearch GPT, data-parallel, 2^19 tokens/step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|ddp|reference]
  (N > 1: torchrun --nproc-per-node N bench.py --gpus N ...; one rank per GPU over NCCL)

Arms:
  ours       the sm_100a engine (tcgen05 GEMMs, fused kernels, flash attention, fused optimizer)
  ddp        plain PyTorch DistributedDataParallel + cuBLAS + SDPA of the same model and optimizer
  ddp-compile  the same under torch.compile, with flex attention (fused sliding window) on every layer
  reference  the upstream project (a TypeScript/TF.js browser trainer; it has no Python package)

Measurement: W untimed warm-up steps, then K timed full training steps (forward, backward, gradient
synchronisation, optimizer) bracketed by a barrier and ``torch.cuda.synchronize()`` on both sides,
timed with CUDA events on the launching stream; the per-step time is the max over ranks. ``value``
uses device-resident synthetic batches; ``e2e`` repeats the measurement through the public
``Trainer.train_step()`` API, which packs each batch on the host, copies it from pinned memory and
reads the loss back every step. SM clocks and throttle reasons are sampled with ``nvidia-smi``
during the timed region. Every step touches tens of GB of activations (far larger than the 126 MB
L2), so no explicit L2 flush is done between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "tokens/s (device-timed, max over ranks)"
def _resident_batches(cfg, rank, world, B, T, accum, device, dtype):
    """Two steps' worth of micro-batches from the configured seeded data stream (the same for both
    arms), kept on the device and alternated in the timed loop."""
    from bitresearch_b200.data.pipeline import make_batch_source
    src = make_batch_source(cfg, "train", rank, world)
    out = []
    for _ in range(2):
        step = []
        for _ in range(accum):
            x, y = src.next(B, T)
            step.append((torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=dtype),
                         torch.from_numpy(np.ascontiguousarray(y)).to(device=device, dtype=dtype)))
        out.append(step)
    return out


def model_desc(m) -> str:
    """e.g. 'autoresearch GPT d512 depth-8 (4x128 heads, vocab 8192, SSSL windows 1024/2048, VE, ReLU^2, QK-norm)'."""
    hd = m.n_embd // m.n_head
    return (f"autoresearch GPT d{m.n_embd} depth-{m.n_layer} ({m.n_head}x{hd} heads, vocab {m.vocab_size}, "
            f"{m.window_pattern} windows {m.sequence_len // 2}/{m.sequence_len}, VE, ReLU^2, QK-norm)")
REF_UNAVAILABLE = ("the reference (gauravsaini/bitresearch) is a TypeScript/TensorFlow.js browser trainer with no "
                   "setup.py/pyproject (pip: 'Directory is not installable'); its GPU path is WebGPU and no Node "
                   "runtime is present")


def _rank_world():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def _max_over_ranks(x: float) -> float:
    if dist.is_initialized():
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def _barrier_sync():
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


def _time_steps(step_fn, K: int, join=None) -> float:
    """ms per step on this rank (CUDA events around K steps). ``join`` makes the launching stream wait for
    work the steps queued on side streams (the parameter exchange that overlaps the next forward), so the
    end event covers all of it."""
    _barrier_sync()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(K):
        step_fn()
    if join is not None:
        join()
    b.record()
    _barrier_sync()
    return a.elapsed_time(b) / K


def _replica_check(params) -> dict:
    """Sum and sum of |x| of every parameter (fp64, per rank), reduced MAX and MIN over ranks: equal
    extremes mean every rank holds bitwise the same values after the timed steps."""
    v = torch.zeros(2, dtype=torch.float64, device="cuda")
    for p in params:
        d = p.detach().double()
        v[0] += d.sum()
        v[1] += d.abs().sum()
    hi, lo = v.clone(), v.clone()
    if dist.is_initialized():
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    return {"replicas_identical": bool(torch.equal(hi, lo)), "param_sum": float(hi[0]), "param_abs_sum": float(hi[1])}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "ddp", "ddp-compile", "reference"])
    ap.add_argument("--preset", default="d512")
    ap.add_argument("--device-batch", type=int, default=0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--comm", default="p2p", choices=["p2p", "nccl"],
                    help="gradient/parameter exchange for N > 1: in-kernel NVLink (p2p) or NCCL")
    ap.add_argument("--gemm-pair", type=int, default=None, choices=[0, 1, 2],
                    help="256-column GEMMs on CTA pairs: 0 none, 1 the default policy (all), 2 all")
    ap.add_argument("overrides", nargs="*")
    args = ap.parse_args()
    rank, world, local = _rank_world()

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": REF_UNAVAILABLE}), flush=True)
        return 0

    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.ops._ext import launch_counts, reset_launch_counts
    from bitresearch_b200.train import Trainer, init_distributed
    from bitresearch_b200.utils.timing import ClockSampler

    torch.cuda.set_device(local)
    if world > 1:
        init_distributed("nccl", timeout_s=300)
    cfg = apply_overrides(preset(args.preset), list(args.overrides))
    if args.device_batch:
        cfg.device_batch = args.device_batch
    cfg.log_every = 0
    cfg.results_tsv = ""
    device = torch.device("cuda", local)
    T = cfg.model.sequence_len
    global_tokens = cfg.total_batch_tokens
    K, W = args.steps, args.warmup

    if args.impl == "ours":
        cfg.impl = "cuda"
        cfg.comm = args.comm
        if args.gemm_pair is not None:
            from bitresearch_b200.ops._ext import ext
            ext().gemm_set_pair(args.gemm_pair)
        tr = Trainer(cfg, device=device, log=lambda m: None)
        tr.initialize()
        accum = tr.grad_accum
        B = tr.device_batch
        batches = _resident_batches(cfg, rank, world, B, T, accum, device, torch.int32)
        it = [0]

        last = [None]

        def step():
            last[0] = tr.train_step(batches[it[0] % 2], sync=False)
            it[0] += 1

        def e2e_step():
            last[0] = tr.train_step()

        def params():
            return list(tr.model.named().values())
    else:
        from baseline.ddp_baseline import DDPBaseline
        cfg.impl = "torch"
        tr = DDPBaseline(cfg, device, compile=args.impl == "ddp-compile")
        accum, B = tr.grad_accum, tr.device_batch
        batches = _resident_batches(cfg, rank, world, B, T, accum, device, torch.int64)
        it = [0]

        last = [None]

        def step():
            last[0] = tr.train_step(batches[it[0] % 2])
            it[0] += 1
        host = [[(x.cpu().pin_memory(), y.cpu().pin_memory()) for x, y in bb] for bb in batches]

        def e2e_step():
            bs = [(x.to(device, non_blocking=True), y.to(device, non_blocking=True)) for x, y in host[it[0] % 2]]
            last[0] = float(tr.train_step(bs))
            it[0] += 1

        def params():
            return list(tr.model.parameters())

    for _ in range(W):
        step()
    clocks = ClockSampler(gpu_index=None).start()
    reset_launch_counts()
    join = tr.join_streams if args.impl == "ours" else None
    ms = _time_steps(step, K, join)
    by_kernel = launch_counts()
    launches = sum(by_kernel.values())
    clk = clocks.stop()
    ms = _max_over_ranks(ms)
    value = global_tokens / (ms / 1e3)

    e2e = None
    if not args.no_e2e:
        for _ in range(1):
            e2e_step()
        ms_e2e = _max_over_ranks(_time_steps(e2e_step, K, join))
        e2e = {"value": global_tokens / (ms_e2e / 1e3), "unit": "tokens/s", "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": 2 * 4 * B * T * accum, "d2h_bytes_per_step": 4,
               "api": "Trainer.train_step()" if args.impl == "ours" else "DDPBaseline.train_step() + loss.item()"}

    # after the timed steps (outside the timed regions): do the ranks hold identical replicas, and the
    # loss of the last step, max over ranks
    check = _replica_check(params())
    final_loss = torch.tensor([float(last[0])], dtype=torch.float64, device="cuda")
    if dist.is_initialized():
        dist.all_reduce(final_loss, op=dist.ReduceOp.MAX)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": (f"synthetic: seeded {cfg.data} stream ({'Zipf(1.1) tokens BOS-packed into geometric-length documents' if cfg.data == 'zipf' else cfg.data}), "
                     "device-timed steps on resident batches, the e2e field through the trainer's pinned pipeline; "
                     "random-init weights"),
            "config": {"model": model_desc(cfg.model), "global_batch": global_tokens, "global_batch_unit": "tokens",
                       "seq_len": T, "device_batch": B, "grad_accum": accum, "parallelism": f"dp{world}",
                       "comm": (args.comm if args.impl == "ours" else "nccl-ddp") if world > 1 else "none",
                       "l2": "inputs larger than L2 (activations tens of GB per step); no flush"},
            "impl": args.impl, "clocks": clk, "e2e": e2e, "final_loss": float(final_loss), **check,
            "gpu_launches": launches if args.impl == "ours" else 0,
            "launches_by_kernel": by_kernel if args.impl == "ours" else {},
        }
        print(json.dumps(line), flush=True)
    if args.impl == "ours":
        tr.destroy()
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
