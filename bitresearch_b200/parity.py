"""Parity bundles: export a reference bundle and validate a model against one.

Bundle layout (the reference's scripts/export_reference.py:64-80, 255-301, read by
scripts/validate_reference_node.ts and src/model/reference.ts):

* ``weights.bin`` + ``weights_meta.json``: fp32 little-endian tensors back to back, C order; the meta maps
  each name to ``{"shape", "offset", "byteLength"}``. Names are the model's variable names, with the
  exporter's ``layer{i}_value_embed`` for value embeddings;
* ``grads.bin`` + ``grads_meta.json``: the gradients of the loss, same layout;
* ``batch.json``: ``{"inputs": [[...]], "targets": [[...]]}``; ``loss.json``: ``{"loss": x}``;
  ``logits.bin``: fp32 [B, T, V].

The reference exporter's model differs from its trainer's model in two places: the value-embedding gate
reads the normalised input instead of the ladder output, and a window of ``ws`` keys spans ``ws + 1``
positions. So a bundle has a ``semantics``: ``exporter`` (what the reference's exporter writes) or
``model`` (gpt.ts). ``export`` records it in an extra ``bundle_meta.json`` (config + semantics); a bundle
without that file is taken as the reference exporter's, on its validation config (src/model/reference.ts:
32-40). The fp32 oracle validates either; the eager model follows gpt.ts, so it validates ``model``
bundles (the reference's own validator compares its model with an ``exporter`` bundle, where the two
quirks make it disagree).

Tolerances are the reference validator's: loss 1e-5, logits and every gradient 1e-4 (absolute).

  python -m bitresearch_b200.parity export --out public/reference [--semantics model|exporter]
  python -m bitresearch_b200.parity validate --bundle public/reference [--impl oracle|torch]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from collections import OrderedDict

import numpy as np
import torch

from .config import GPTConfig
from .models.reference import reference_forward

VALIDATION_CONFIG = GPTConfig(vocab_size=8192, n_layer=4, n_head=4, n_kv_head=4, n_embd=256, sequence_len=256,
                              window_pattern="SSSL")
TOL = {"loss": 1e-5, "logits": 1e-4, "grads": 1e-4}


def _bundle_name(name: str) -> str:
    return f"layer{name[3:]}_value_embed" if name.startswith("ve_") else name


def _model_name(name: str) -> str:
    if name.endswith("_value_embed"):
        return f"ve_{name[len('layer'):-len('_value_embed')]}"
    return name


def write_tensors(meta_path: str, bin_path: str, tensors: "OrderedDict[str, torch.Tensor]") -> None:
    meta, off = {}, 0
    with open(bin_path, "wb") as f:
        for name, t in tensors.items():
            a = np.ascontiguousarray(t.detach().cpu().float().numpy(), dtype="<f4")
            meta[name] = {"shape": list(a.shape), "offset": off, "byteLength": int(a.nbytes)}
            f.write(a.tobytes())
            off += a.nbytes
    with open(meta_path, "w") as f:
        json.dump(meta, f, indent=2)
        f.write("\n")


def read_tensors(meta_path: str, bin_path: str) -> "OrderedDict[str, torch.Tensor]":
    with open(meta_path) as f:
        meta = json.load(f)
    buf = np.fromfile(bin_path, dtype=np.uint8)
    out = OrderedDict()
    for name, m in meta.items():
        shape, off, nb = list(m["shape"]), int(m["offset"]), int(m["byteLength"])
        if nb != int(np.prod(shape)) * 4:
            raise ValueError(f"{name}: byteLength {nb} does not match shape {shape}")
        if off < 0 or off + nb > buf.size:
            raise ValueError(f"{name}: bytes [{off}, {off + nb}) outside {os.path.basename(bin_path)} ({buf.size})")
        out[name] = torch.from_numpy(buf[off:off + nb].view("<f4").reshape(shape).copy())
    return out


def coverage(specs: list[tuple[str, tuple]], tensors: dict) -> dict:
    """Which model variables a bundle covers: missing, extra and shape-mismatched names (the reference's
    summarizeReferenceCoverage, src/model/reference.ts:78-132)."""
    names = {_model_name(n): t for n, t in tensors.items()}
    want = {n: tuple(s) for n, s in specs}
    missing = sorted(n for n in want if n not in names)
    extra = sorted(n for n in names if n not in want)
    bad = sorted(n for n in want if n in names and tuple(names[n].shape) != want[n])
    return {"missing": missing, "extra": extra, "shape_mismatch": bad, "complete": not (missing or extra or bad)}


def _quirks(semantics: str) -> dict:
    if semantics not in ("exporter", "model"):
        raise ValueError(f"semantics must be 'exporter' or 'model', got {semantics!r}")
    ex = semantics == "exporter"
    return {"gate_from_prenorm": ex, "exporter_window": ex}


def export_bundle(out_dir: str, cfg: GPTConfig = VALIDATION_CONFIG, batch_size: int = 2, seed: int = 100,
                  semantics: str = "model", weight_seed: int = 42) -> float:
    """Writes a bundle from the fp32 oracle (weights N(0, 0.02) from ``weight_seed``, batch from ``seed``);
    returns the loss."""
    from .models.gpt import GPT
    os.makedirs(out_dir, exist_ok=True)
    model = GPT(cfg, init="normal", seed=weight_seed)
    params = OrderedDict((n, p.detach().clone().requires_grad_(True)) for n, p in model.named().items())
    g = torch.Generator().manual_seed(seed)
    inputs = torch.randint(0, cfg.vocab_size, (batch_size, cfg.sequence_len), generator=g)
    targets = torch.randint(0, cfg.vocab_size, (batch_size, cfg.sequence_len), generator=g)
    logits, loss = reference_forward(params, cfg, inputs, targets, **_quirks(semantics))
    loss.backward()
    write_tensors(os.path.join(out_dir, "weights_meta.json"), os.path.join(out_dir, "weights.bin"),
                  OrderedDict((_bundle_name(n), p) for n, p in params.items()))
    write_tensors(os.path.join(out_dir, "grads_meta.json"), os.path.join(out_dir, "grads.bin"),
                  OrderedDict((_bundle_name(n), p.grad) for n, p in params.items()))
    with open(os.path.join(out_dir, "batch.json"), "w") as f:
        json.dump({"inputs": inputs.tolist(), "targets": targets.tolist()}, f)
    with open(os.path.join(out_dir, "loss.json"), "w") as f:
        json.dump({"loss": float(loss.item())}, f)
    logits.detach().float().numpy().astype("<f4").tofile(os.path.join(out_dir, "logits.bin"))
    with open(os.path.join(out_dir, "bundle_meta.json"), "w") as f:
        json.dump({"config": cfg.to_reference_dict(), "semantics": semantics}, f)
    return float(loss.item())


def load_bundle(bundle_dir: str):
    """(config, semantics, weights, grads, inputs, targets, loss, logits)."""
    meta_path = os.path.join(bundle_dir, "bundle_meta.json")
    if os.path.isfile(meta_path):
        with open(meta_path) as f:
            m = json.load(f)
        cfg, semantics = GPTConfig.from_reference_dict(m["config"]), m["semantics"]
    else:  # written by the reference's exporter
        cfg, semantics = VALIDATION_CONFIG, "exporter"
    weights = read_tensors(os.path.join(bundle_dir, "weights_meta.json"), os.path.join(bundle_dir, "weights.bin"))
    grads = read_tensors(os.path.join(bundle_dir, "grads_meta.json"), os.path.join(bundle_dir, "grads.bin"))
    with open(os.path.join(bundle_dir, "batch.json")) as f:
        batch = json.load(f)
    with open(os.path.join(bundle_dir, "loss.json")) as f:
        loss = float(json.load(f)["loss"])
    inputs = torch.tensor(batch["inputs"], dtype=torch.int64)
    targets = torch.tensor(batch["targets"], dtype=torch.int64)
    if inputs.ndim != 2 or inputs.shape[1] != cfg.sequence_len or targets.shape != inputs.shape:
        raise ValueError(f"batch.json: inputs/targets must both be [B, {cfg.sequence_len}]")
    logits = torch.from_numpy(np.fromfile(os.path.join(bundle_dir, "logits.bin"), dtype="<f4"))
    logits = logits.view(inputs.shape[0], cfg.sequence_len, cfg.vocab_size)
    return cfg, semantics, weights, grads, inputs, targets, loss, logits


def validate_bundle(bundle_dir: str, impl: str = "oracle", semantics: str | None = None) -> dict:
    """Recomputes loss, logits and gradients from the bundle's weights and batch with ``impl`` ('oracle':
    the fp32 restatement with the bundle's semantics; 'torch': the eager model) and compares them with the
    bundle. Returns a report with ``ok``, the differences and the coverage."""
    from .models.gpt import GPT
    cfg, sem, weights, grads, inputs, targets, loss_ref, logits_ref = load_bundle(bundle_dir)
    sem = semantics or sem
    model = GPT(cfg, init="normal", seed=0)
    specs = [(n, tuple(p.shape)) for n, p in model.named().items()]
    cov = coverage(specs, weights)
    gcov = coverage(specs, grads)
    report = {"impl": impl, "semantics": sem, "coverage": cov, "grads_coverage": gcov}
    if not (cov["complete"] and gcov["complete"]):
        report["ok"] = False
        return report
    w = {_model_name(n): t for n, t in weights.items()}
    gref = {_model_name(n): t for n, t in grads.items()}
    if impl == "oracle":
        params = {n: w[n].clone().requires_grad_(True) for n, _ in specs}
        logits, loss = reference_forward(params, cfg, inputs, targets, **_quirks(sem))
        loss.backward()
        got = {n: p.grad for n, p in params.items()}
    elif impl == "torch":
        with torch.no_grad():
            for n, p in model.named().items():
                p.copy_(w[n])
        loss = model.forward_torch(inputs, targets)
        loss.backward()
        got = {n: p.grad for n, p in model.named().items()}
        with torch.no_grad():
            logits = model.forward_torch(inputs)
    else:
        raise ValueError(f"impl must be 'oracle' or 'torch', got {impl!r}")
    report["loss"] = {"ours": float(loss.item()), "bundle": loss_ref, "diff": abs(float(loss.item()) - loss_ref)}
    report["logits_max_diff"] = float((logits.detach().float() - logits_ref).abs().max())
    report["grads_max_diff"] = {n: float((got[n].float() - gref[n]).abs().max()) for n, _ in specs}
    report["ok"] = (report["loss"]["diff"] <= TOL["loss"] and report["logits_max_diff"] <= TOL["logits"]
                    and max(report["grads_max_diff"].values()) <= TOL["grads"])
    return report


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="export / validate parity bundles")
    sub = ap.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("export")
    e.add_argument("--out", default=os.path.join("public", "reference"))
    e.add_argument("--semantics", default="model", choices=["model", "exporter"])
    e.add_argument("--batch-size", type=int, default=2)
    e.add_argument("--seed", type=int, default=100)
    e.add_argument("--config", default="", help="JSON of the model config (reference field names)")
    v = sub.add_parser("validate")
    v.add_argument("--bundle", default=os.path.join("public", "reference"))
    v.add_argument("--impl", default="oracle", choices=["oracle", "torch"])
    v.add_argument("--semantics", default=None, choices=["model", "exporter"])
    args = ap.parse_args(argv)
    if args.cmd == "export":
        cfg = GPTConfig.from_reference_dict(json.loads(args.config)) if args.config else VALIDATION_CONFIG
        loss = export_bundle(args.out, cfg, args.batch_size, args.seed, args.semantics)
        print(f"exported {args.semantics} bundle to {args.out}; loss {loss:.8f}")
        return 0
    r = validate_bundle(args.bundle, args.impl, args.semantics)
    for key in ("coverage", "grads_coverage"):
        c = r[key]
        print(f"{key}: complete={c['complete']} missing={c['missing']} extra={c['extra']} "
              f"shape_mismatch={c['shape_mismatch']}")
    if "loss" in r:
        worst = max(r["grads_max_diff"].items(), key=lambda kv: kv[1])
        print(f"loss ours {r['loss']['ours']:.8f} bundle {r['loss']['bundle']:.8f} (diff {r['loss']['diff']:.2e}, "
              f"tol {TOL['loss']}); logits max diff {r['logits_max_diff']:.2e}; worst grad {worst[0]} "
              f"{worst[1]:.2e} (tol {TOL['grads']})")
    print("PASS" if r["ok"] else "FAIL")
    return 0 if r["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
