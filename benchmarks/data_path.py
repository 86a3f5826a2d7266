"""Host data-path throughput: the native packer per synthetic source, and BPE encoding of a synthetic
web-like text corpus on one thread and on a thread pool.

  python benchmarks/data_path.py [--docs 20000] [--workers 8]

Every number is host wall time (no GPU involved). A training step needs its batches at the device's
rate, e.g. 2^19 tokens per step in about 0.2 s on one GPU (2.6M tokens/s); the packer runs on a
prefetch thread with the GIL released.
"""
from __future__ import annotations

import argparse
import os
import random
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def packer(batches: int = 8) -> None:
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.data.pipeline import make_batch_source
    for data in ("zipf", "markov", "uniform"):
        cfg = apply_overrides(preset("d512"), [f"data={data}"])
        src = make_batch_source(cfg, "train", 0, 1)
        src.next(128, 2048)
        t = time.perf_counter()
        for _ in range(batches):
            src.next(128, 2048)
        dt = time.perf_counter() - t
        print(f"packer {data:8s}: {batches * 128 * 2048 / dt / 1e6:6.2f} M tokens/s (128 x 2048 batches)")


def bpe(n_docs: int, workers: int) -> None:
    from bitresearch_b200.data.tokenizer import BPETokenizer
    rng = random.Random(0)
    words = ["".join(rng.choice("abcdefghijklmnopqrstuvwxyz") for _ in range(rng.randint(1, 10))) for _ in range(5000)]
    # web text is mostly ASCII with curly quotes, dashes, accents and some other scripts mixed in
    words += ["\u201cquote\u201d", "caf\u00e9", "na\u00efve", "\u2014", "\u4f60\u597d", "it\u2019s", "\u00bd"] * 40
    docs = [" ".join(rng.choice(words) for _ in range(rng.randint(20, 400))) + "." for _ in range(n_docs)]
    mb = sum(map(len, docs)) / 1e6
    t = time.perf_counter()
    tok = BPETokenizer().train(docs[:5000], 4096)
    print(f"bpe train: {time.perf_counter() - t:.2f} s (5000 docs, 4096 tokens)")
    t = time.perf_counter()
    for d in docs:
        tok._enc.encode_chunks(tok._re.findall(d))
    with_regex = mb / (time.perf_counter() - t)
    t = time.perf_counter()
    tok.batch_encode(docs)
    serial = mb / (time.perf_counter() - t)
    with tok.pool(workers) as pool:
        tok.batch_encode(docs[:500], pool=pool)  # workers started
        t = time.perf_counter()
        tok.batch_encode(docs, pool=pool)
        pooled = mb / (time.perf_counter() - t)
    print(f"bpe encode: {serial:.1f} MB/s on one thread (regex split: {with_regex:.1f}), {pooled:.1f} MB/s on "
          f"{workers} threads ({mb:.1f} MB)")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--docs", type=int, default=20000)
    ap.add_argument("--workers", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    packer()
    bpe(args.docs, args.workers)
    return 0


if __name__ == "__main__":
    sys.exit(main())
