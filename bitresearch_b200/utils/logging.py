"""Run summaries, ``results.tsv`` and JSONL metrics.

* ``summary_block`` prints the autoresearch summary (src/distributed/trainer.ts:1059-1068, format of
  program.md:125-136) so ``grep '^val_bpb:'`` works on the log.
* ``ResultsLogger`` appends ``commit val_bpb memory_gb status description`` rows
  (src/train/results-logger.ts:29-97).
* ``MetricsLog`` writes one JSON object per step (replaces the reference's Chart.js dashboard).
"""
from __future__ import annotations

import json
import os
import subprocess
from dataclasses import asdict, dataclass, field

TSV_HEADER = "commit\tval_bpb\tmemory_gb\tstatus\tdescription"


@dataclass
class TrainerMetrics:
    """Fields of the reference's ``TrainerMetrics`` (trainer.ts:52-67)."""

    step: int = 0
    loss: float = 0.0
    smooth_loss: float = 0.0
    grad_norm: float = 0.0
    tokens_per_sec: float = 0.0
    total_tokens: int = 0
    peers_connected: int = 1
    all_reduce_time_ms: float = 0.0
    compute_time_ms: float = 0.0
    step_time_ms: float = 0.0
    elapsed_seconds: float = 0.0
    val_bpb: float = 0.0
    mfu_percent: float = 0.0
    num_params_m: float = 0.0
    skipped_steps: int = 0
    extra: dict = field(default_factory=dict)

    def to_dict(self):
        return asdict(self)


def summary_block(m: TrainerMetrics, training_seconds: float, total_seconds: float, peak_vram_mb: float,
                  depth: int) -> str:
    # synthetic Markov data knows its own loss floor; it follows the reference's fields as an extra line
    floor = [f"val_bpb_floor:    {m.extra['val_bpb_floor']:.6f}"] if "val_bpb_floor" in m.extra else []
    return "\n".join([
        "---",
        f"val_bpb:          {m.val_bpb:.6f}",
        f"training_seconds: {training_seconds:.1f}",
        f"total_seconds:    {total_seconds:.1f}",
        f"peak_vram_mb:     {peak_vram_mb:.1f}",
        f"mfu_percent:      {m.mfu_percent:.2f}",
        f"total_tokens_M:   {m.total_tokens / 1e6:.1f}",
        f"num_steps:        {m.step}",
        f"num_params_M:     {m.num_params_m:.1f}",
        f"depth:            {depth}",
    ] + floor)


def git_commit_short() -> str:
    try:
        return subprocess.check_output(["git", "rev-parse", "--short=7", "HEAD"], text=True,
                                       stderr=subprocess.DEVNULL).strip()
    except Exception:
        return "unknown"


class ResultsLogger:
    def __init__(self, path: str = "results.tsv"):
        self.path = os.path.abspath(path)
        if not os.path.exists(self.path):
            with open(self.path, "w") as f:
                f.write(TSV_HEADER + "\n")
        else:
            with open(self.path) as f:
                content = f.read()
            if not content.startswith("commit\t"):
                with open(self.path, "w") as f:
                    f.write(TSV_HEADER + "\n" + content)

    def log(self, val_bpb: float, peak_memory_mb: float, status: str, description: str, commit: str | None = None):
        commit = commit or git_commit_short()
        vb = "0.000000" if status == "crash" else f"{val_bpb:.6f}"
        mem = "0.0" if status == "crash" else f"{peak_memory_mb / 1024:.1f}"
        desc = " ".join(description.replace("\t", " ").splitlines()).strip()
        with open(self.path, "a") as f:
            f.write(f"{commit}\t{vb}\t{mem}\t{status}\t{desc}\n")

    def read_all(self) -> list[dict]:
        with open(self.path) as f:
            lines = f.read().strip().split("\n")[1:]
        out = []
        for line in lines:
            parts = line.split("\t")
            if len(parts) < 4:
                continue
            out.append({"commit": parts[0], "val_bpb": float(parts[1] or 0), "memory_gb": float(parts[2] or 0),
                        "status": parts[3], "description": "\t".join(parts[4:])})
        return out

    def best_bpb(self) -> float:
        keep = [r["val_bpb"] for r in self.read_all() if r["status"] == "keep"]
        return min(keep) if keep else float("inf")


class MetricsLog:
    def __init__(self, path: str):
        self.path = path
        if path:
            d = os.path.dirname(path)
            if d:
                os.makedirs(d, exist_ok=True)

    def write(self, obj: dict) -> None:
        if self.path:
            with open(self.path, "a") as f:
                f.write(json.dumps(obj) + "\n")
