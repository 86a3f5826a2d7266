"""``.safetensors`` checkpoints with the reference trainer's tensor names.

Format (src/distributed/trainer.ts:1102-1166): ``[u64 LE header length][JSON header][raw data]``;
every tensor is ``F32`` keyed by its variable name, in ``getTrainableVariables`` order, and
``__metadata__`` carries step, lossScale, totalTokens and the model config as JSON.

Differences from the reference, on purpose:

* ``__metadata__`` values are strings, as the safetensors specification requires (the reference
  writes numbers, trainer.ts:1132-1137), so the ``safetensors`` library can read these files.
* Optimizer state is saved as extra tensors (``adam_m_*``, ``adam_v_*``, ``muon_mom_*``,
  ``muon_sec_*``, the names of muon.ts:389-402) plus per-parameter step counters and the schedule
  state (``totalTrainingTime``, ``smoothLoss``) in metadata; the reference saves none of them.
* Loading accepts the parity exporter's ``layer{i}_value_embed`` alias for ``ve_{i}``
  (scripts/export_reference.py:168) and, like trainer.ts:1244-1255, only warns on missing names.
* ``save_sharded``: each data-parallel rank writes the tensors it owns; ``merge_shards`` joins them.
"""
from __future__ import annotations

import json
import os
import re
import struct
import time
from collections import OrderedDict
from typing import Mapping

import numpy as np
import torch

_DTYPES = {torch.float32: ("F32", np.float32), torch.bfloat16: ("BF16", None), torch.float16: ("F16", np.float16),
           torch.int32: ("I32", np.int32), torch.int64: ("I64", np.int64)}
_NP = {"F32": np.float32, "F16": np.float16, "I32": np.int32, "I64": np.int64}


def checkpoint_filename(step: int) -> str:
    """``checkpoint_step{NNNNNN}_{ISO}.safetensors`` (trainer.ts:1106-1107)."""
    ts = time.strftime("%Y-%m-%dT%H-%M-%S", time.gmtime())
    return f"checkpoint_step{step:06d}_{ts}.safetensors"


def to_bytes(tensors: Mapping[str, torch.Tensor], metadata: Mapping[str, object] | None = None) -> bytes:
    header: "OrderedDict[str, object]" = OrderedDict()
    blobs = []
    off = 0
    for name, t in tensors.items():
        t = t.detach().to("cpu").contiguous()
        if t.dtype == torch.bfloat16:
            raw = t.view(torch.int16).numpy().tobytes()
            dt = "BF16"
        else:
            if t.dtype not in _DTYPES:
                t = t.float()
            dt = _DTYPES[t.dtype][0]
            raw = t.numpy().tobytes()
        header[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {k: (v if isinstance(v, str) else json.dumps(v)) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)  # keep the data section 8-byte aligned
    return struct.pack("<Q", len(hb)) + hb + b"".join(blobs)


def from_bytes(buf: bytes) -> tuple["OrderedDict[str, torch.Tensor]", dict[str, str]]:
    (hlen,) = struct.unpack("<Q", buf[:8])
    header = json.loads(buf[8:8 + hlen].decode())
    base = 8 + hlen
    meta = header.pop("__metadata__", {}) or {}
    out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    for name, e in header.items():
        a, b = e["data_offsets"]
        raw = buf[base + a: base + b]
        if e["dtype"] == "BF16":
            t = torch.frombuffer(bytearray(raw), dtype=torch.int16).view(torch.bfloat16)
        else:
            t = torch.from_numpy(np.frombuffer(raw, dtype=_NP[e["dtype"]]).copy())
        out[name] = t.reshape(e["shape"])
    return out, {k: (v if isinstance(v, str) else json.dumps(v)) for k, v in meta.items()}


def save(path: str, tensors: Mapping[str, torch.Tensor], metadata: Mapping[str, object] | None = None) -> str:
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(to_bytes(tensors, metadata))
    os.replace(tmp, path)
    return path


def load(path: str):
    with open(path, "rb") as f:
        return from_bytes(f.read())


_ALIAS = re.compile(r"^layer(\d+)_value_embed$")


def canonical_name(name: str) -> str:
    m = _ALIAS.match(name)
    return f"ve_{m.group(1)}" if m else name


def build_state(model, optimizer=None, *, step: int, loss_scale: float = 1.0, total_tokens: int = 0,
                extra_meta: Mapping[str, object] | None = None, owned: set | None = None):
    """Tensors + metadata for a checkpoint (model weights in reference order, then optimizer)."""
    tensors: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    for name, p in model.named().items():
        if owned is None or name in owned:
            tensors[name] = p.detach().float()
    meta: dict[str, object] = {
        "step": str(step),
        "lossScale": str(loss_scale),
        "totalTokens": str(total_tokens),
        "config": json.dumps(model.cfg.to_reference_dict()),
    }
    if optimizer is not None:
        for k, t in optimizer.state_tensors().items():
            tensors[k] = t.detach().float()
        meta["optimizer_steps"] = json.dumps(optimizer.state_steps())
    if extra_meta:
        for k, v in extra_meta.items():
            meta[k] = v if isinstance(v, str) else json.dumps(v)
    return tensors, meta


def restore(model, tensors: Mapping[str, torch.Tensor], meta: Mapping[str, str], optimizer=None, log=print) -> dict:
    """Assign weights by name; returns the parsed metadata. Missing names only warn."""
    named = model.named()
    by_canon = {canonical_name(k): v for k, v in tensors.items()}
    restored = 0
    with torch.no_grad():
        for name, p in named.items():
            t = by_canon.get(name)
            if t is None:
                log(f"warning: no checkpoint data for weight: {name}")
                continue
            p.copy_(t.to(device=p.device, dtype=p.dtype).view_as(p))
            restored += 1
    info: dict[str, object] = {"restored": restored}
    for k in ("step", "lossScale", "totalTokens"):
        if k in meta:
            info[k] = json.loads(meta[k])
    for k, v in meta.items():
        if k not in info:
            try:
                info[k] = json.loads(v)
            except (TypeError, ValueError):
                info[k] = v
    if optimizer is not None:
        steps = info.get("optimizer_steps") or {}
        info["optimizer_loaded"] = optimizer.load_state(dict(tensors), steps)
    return info


def save_sharded(dirpath: str, rank: int, world: int, tensors, meta) -> str:
    meta = dict(meta)
    meta["shard"] = f"{rank}/{world}"
    return save(os.path.join(dirpath, f"shard_{rank:05d}_of_{world:05d}.safetensors"), tensors, meta)


def merge_shards(dirpath: str, out_path: str, order: list[str] | None = None) -> str:
    files = sorted(f for f in os.listdir(dirpath) if f.startswith("shard_") and f.endswith(".safetensors"))
    merged: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    meta: dict[str, str] = {}
    opt_steps: dict = {}
    for f in files:
        t, m = load(os.path.join(dirpath, f))
        merged.update(t)
        if "optimizer_steps" in m:
            opt_steps.update(json.loads(m["optimizer_steps"]))
        for k, v in m.items():
            meta.setdefault(k, v)
    meta.pop("shard", None)
    if opt_steps:
        meta["optimizer_steps"] = json.dumps(opt_steps)
    if order:
        rest = [k for k in merged if k not in order]
        merged = OrderedDict((k, merged[k]) for k in [*order, *rest] if k in merged)
    return save(out_path, merged, meta)
