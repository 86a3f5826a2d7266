"""The reference's ring all-reduce over a ``torch.distributed`` process group.

Algorithm (src/distributed/ring-allreduce.ts:85-215): the flat buffer is split into N chunks of
``ceil(P/N)`` elements; N-1 reduce-scatter steps send chunk ``(r - s) mod N`` to the right neighbour
and add the chunk ``(r - s - 1) mod N`` received from the left; then N-1 all-gather steps forward
fully-reduced chunks. The wire payload may be f16 (webrtc-mesh.ts:562, 510-511) or bf16/fp32.

Fix relative to the reference: after the reduce-scatter rank r holds the full sum of chunk
``(r + 1) mod N``; the reference divides chunk r instead (ring-allreduce.ts:161-165), which is
overwritten during the all-gather, so it returns the SUM. Here the owned chunk is scaled by 1/N and
the result is the mean.

Failure handling mirrors the reference's abort-and-skip: a receive that does not complete within
``timeout_s`` aborts the operation and ``all_reduce`` returns ``None`` (ring-allreduce.ts:236-265);
the caller skips the optimizer update. Every message carries (step, phase, chunk) in a small header
tensor so a late chunk from an earlier step is detected instead of being consumed (the reference keys
chunks only by index, ring-allreduce.ts:225).

This path is for CPU/gloo worlds and as the algorithmic oracle; on NVSwitch the in-kernel
reduce-scatter/all-gather of :mod:`bitresearch_b200.parallel.comm` replaces it.
"""
from __future__ import annotations

import datetime
import math

import torch
import torch.distributed as dist

_WIRE = {"fp16": torch.float16, "f16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32,
         "f32": torch.float32}


class RingAllReduce:
    def __init__(self, group=None, wire_dtype: str = "fp16", timeout_s: float = 10.0, on_progress=None, log=None,
                 elastic=None):
        self.group = group
        self.elastic = elastic  # an ElasticGroup: ranks are ring positions, sends go through its gloo group
        self.wire = _WIRE[wire_dtype]
        self.timeout_s = timeout_s
        self.on_progress = on_progress
        self.log = log or (lambda m: None)
        self.aborted = False

    def abort(self, reason: str) -> None:
        self.aborted = True
        self.log(f"all-reduce aborted: {reason}")

    def _wait(self, work) -> bool:
        try:
            return bool(work.wait(timeout=datetime.timedelta(seconds=self.timeout_s)))
        except Exception as e:  # gloo raises on timeout / peer loss
            self.log(f"wait failed: {e}")
            return False

    def all_reduce(self, flat: torch.Tensor, step_id: int = 0) -> torch.Tensor | None:
        """Mean of ``flat`` over the group; ``None`` if aborted. ``flat`` is not modified."""
        if self.elastic is None and not dist.is_initialized():
            return flat.clone()
        N = self.elastic.size if self.elastic is not None else dist.get_world_size(self.group)
        if N <= 1:
            return flat.clone()
        self.aborted = False
        if self.elastic is not None:
            r = self.elastic.rank
            right, left = (r + 1) % N, (r - 1) % N
            isend, irecv = self.elastic.isend, self.elastic.irecv
        else:
            r = dist.get_rank(self.group)
            ranks = dist.get_process_group_ranks(self.group) if self.group is not None else list(range(N))
            right, left = ranks[(r + 1) % N], ranks[(r - 1) % N]
            isend = lambda t, d: dist.isend(t, d, group=self.group)  # noqa: E731
            irecv = lambda t, s: dist.irecv(t, s, group=self.group)  # noqa: E731
        P = flat.numel()
        cs = math.ceil(P / N)
        work = torch.zeros(N * cs, dtype=torch.float32)
        work[:P] = flat.detach().float().cpu()
        chunks = work.view(N, cs)
        hdr_out = torch.zeros(3, dtype=torch.int64)
        hdr_in = torch.zeros(3, dtype=torch.int64)
        buf_in = torch.empty(cs, dtype=self.wire)

        def exchange(send_idx: int, recv_idx: int, phase: int) -> torch.Tensor | None:
            hdr_out[0], hdr_out[1], hdr_out[2] = step_id, phase, send_idx
            payload = chunks[send_idx].to(self.wire)
            try:
                reqs = [isend(hdr_out, right), isend(payload, right)]
                rh = irecv(hdr_in, left)
                rb = irecv(buf_in, left)
            except Exception as e:  # a closed connection to a lost peer can raise at post time
                self.log(f"send/recv failed: {e}")
                return None
            if not (self._wait(rh) and self._wait(rb)):
                return None
            for q in reqs:
                if not self._wait(q):
                    return None
            if int(hdr_in[0]) != step_id or int(hdr_in[1]) != phase or int(hdr_in[2]) != recv_idx:
                self.log(f"unexpected chunk header {hdr_in.tolist()} (want {[step_id, phase, recv_idx]})")
                return None
            return buf_in.float()

        for s in range(N - 1):
            got = exchange((r - s) % N, (r - s - 1) % N, 0)
            if got is None:
                self.abort(f"timeout at scatter step {s}")
                return None
            chunks[(r - s - 1) % N] += got
            if self.on_progress:
                self.on_progress("scatter", s + 1, N - 1)
        owned = (r + 1) % N
        chunks[owned] /= N
        # the owned chunk goes on the wire again in the gather phase; round it once so every rank ends
        # with bit-identical values (the owner would otherwise keep the unrounded copy)
        chunks[owned] = chunks[owned].to(self.wire).float()
        for s in range(N - 1):
            got = exchange((r - s + 1) % N, (r - s) % N, 1)
            if got is None:
                self.abort(f"timeout at gather step {s}")
                return None
            chunks[(r - s) % N] = got
            if self.on_progress:
                self.on_progress("gather", s + 1, N - 1)
        return work[:P].to(flat.device).view_as(flat)
