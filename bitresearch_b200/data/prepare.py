"""Data preparation: train the BPE tokenizer, tokenize text shards into BOS-prefixed .bin shards, and
mirror everything into a parity directory with a manifest the trainer can discover.

  python -m bitresearch_b200.data.prepare [--cache-dir ~/.cache/autoresearch] [--public-data-dir public/data]

Steps and layout follow scripts/prepare_wasm.ts:229-311 and scripts/parity-artifacts.ts:47-137:

* input: ``<cache>/text/*.txt``, one document per line (empty lines skipped); shards whose name
  contains ``06542`` are the validation split;
* training corpus: the training shards in name order (``--train-shards`` caps the count), each
  document cut to ``--train-doc-cap`` characters, stopping once ``--train-max-chars`` are collected;
* tokenizer: byte-level BPE with ``--vocab-size - 4`` base tokens and four reserved specials, saved
  as ``<tokenizer>/tokenizer.json`` and ``token_bytes.bin``;
* shards: every text shard (``--tokenize-shards`` caps the count) to ``<bin>/<name>.bin``: int32 ids,
  each document preceded by BOS (the first special token);
* parity mirror: ``<public>/parity/{bin,tokenizer}/`` copies, ``<public>/parity/manifest.json``, and
  the legacy entry points ``<public>/{tokens.bin,token_bytes.bin,tokenizer.json,tokens_meta.json}``
  (the first training shard becomes ``tokens.bin``).

The environment knobs of the reference script are honoured as defaults: PREPARE_WASM_OUTPUT_DIR,
PREPARE_WASM_TOKENIZER_DIR, PREPARE_WASM_TRAIN_SHARDS, PREPARE_WASM_TRAIN_MAX_CHARS,
PREPARE_WASM_TRAIN_DOC_CAP, PREPARE_WASM_TOKENIZE_SHARDS.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import time

import numpy as np

from .tokenizer import DEFAULT_VOCAB_SIZE, SPECIAL_TOKENS, BPETokenizer

VAL_SHARD_MARK = "06542"


def _env_int(name: str, default: int, minimum: int) -> int:
    raw = os.environ.get(name, "")
    if raw == "":
        return default
    v = int(raw)
    if v < minimum:
        raise ValueError(f"{name} must be >= {minimum}")
    return v


def collect_training_corpus(text_dir: str, files: list[str], max_chars: int, doc_cap: int,
                            log=print) -> tuple[list[str], int]:
    docs: list[str] = []
    chars = 0
    for name in files:
        with open(os.path.join(text_dir, name), encoding="utf-8") as f:
            for line in f:
                line = line.rstrip("\n")
                if not line:
                    continue
                doc = line[:doc_cap]
                docs.append(doc)
                chars += len(doc)
                if chars >= max_chars:
                    log(f"reached the training character cap at {chars:,} characters")
                    return docs, chars
    return docs, chars


def tokenize_shard(tok: BPETokenizer, src: str, dst: str, batch: int = 2048, pool=None) -> tuple[int, int]:
    """Writes BOS-prefixed int32 ids of every non-empty line of ``src`` to ``dst`` (atomically); with a
    ``pool`` (``tok.pool(n)``) each batch of lines is encoded across its threads, in order."""
    if pool is not None:
        batch = max(batch, 16384)  # enough 256-line tasks per flush to keep every worker busy
    tmp = dst + ".tmp"
    docs = toks = 0
    bos = np.array([tok.bos_id], dtype=np.int32)
    try:
        with open(src, encoding="utf-8") as f, open(tmp, "wb") as out:
            pending: list[str] = []

            def flush():
                nonlocal docs, toks
                for ids in tok.batch_encode(pending, pool=pool):
                    bos.tofile(out)
                    np.asarray(ids, dtype=np.int32).tofile(out)
                    toks += 1 + len(ids)
                docs += len(pending)
                pending.clear()

            for line in f:
                line = line.rstrip("\n")
                if line:
                    pending.append(line)
                    if len(pending) >= batch:
                        flush()
            flush()
        os.replace(tmp, dst)
    except BaseException:
        if os.path.exists(tmp):
            os.remove(tmp)
        raise
    return docs, toks


def sync_parity_artifacts(cache_dir: str, bin_dir: str, tokenizer_dir: str, public_dir: str) -> str:
    """Mirrors shards and tokenizer into ``<public>/parity`` and writes its manifest; returns the path."""
    parity = os.path.join(public_dir, "parity")
    pbin, ptok = os.path.join(parity, "bin"), os.path.join(parity, "tokenizer")
    bins = sorted(f for f in os.listdir(bin_dir) if f.endswith(".bin") and os.path.isfile(os.path.join(bin_dir, f)))
    if not bins:
        raise FileNotFoundError(f"no .bin artifacts in {bin_dir}")
    tok_files = ["token_bytes.bin", "tokenizer.json"]
    for name in tok_files:
        if not os.path.isfile(os.path.join(tokenizer_dir, name)):
            raise FileNotFoundError(os.path.join(tokenizer_dir, name))
    for d in (pbin, ptok):
        shutil.rmtree(d, ignore_errors=True)
        os.makedirs(d)
    for name in bins:
        shutil.copyfile(os.path.join(bin_dir, name), os.path.join(pbin, name))
    for name in tok_files:
        shutil.copyfile(os.path.join(tokenizer_dir, name), os.path.join(pbin, name))
        shutil.copyfile(os.path.join(tokenizer_dir, name), os.path.join(ptok, name))
    manifest = {
        "cacheDir": cache_dir,
        "publicDataDir": public_dir,
        "parityUrl": "/data/parity",
        "binUrl": "/data/parity/bin",
        "tokenizerUrl": "/data/parity/tokenizer",
        "source": {"binDir": bin_dir, "tokenizerDir": tokenizer_dir},
        "files": {"bin": bins, "tokenizer": tok_files},
    }
    mpath = os.path.join(parity, "manifest.json")
    with open(mpath, "w") as f:
        f.write(json.dumps(manifest, indent=2) + "\n")
    # legacy root entry points: the first non-validation shard becomes tokens.bin
    default_bin = next((b for b in bins if VAL_SHARD_MARK not in b), bins[0])
    shutil.copyfile(os.path.join(bin_dir, default_bin), os.path.join(public_dir, "tokens.bin"))
    shutil.copyfile(os.path.join(tokenizer_dir, "token_bytes.bin"), os.path.join(public_dir, "token_bytes.bin"))
    shutil.copyfile(os.path.join(tokenizer_dir, "tokenizer.json"), os.path.join(public_dir, "tokenizer.json"))
    with open(os.path.join(tokenizer_dir, "tokenizer.json")) as f:
        meta = json.load(f)
    tokens_meta = {
        "source": default_bin,
        "numTokens": os.path.getsize(os.path.join(bin_dir, default_bin)) // 4,
        "vocabSize": meta.get("fullVocabSize", meta.get("vocabSize")),
        "parityManifest": "/data/parity/manifest.json",
    }
    with open(os.path.join(public_dir, "tokens_meta.json"), "w") as f:
        f.write(json.dumps(tokens_meta, indent=2) + "\n")
    return mpath


def main(argv=None) -> int:
    home_cache = os.path.join(os.path.expanduser("~"), ".cache", "autoresearch")
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--cache-dir", default=home_cache)
    ap.add_argument("--text-dir", default="")
    ap.add_argument("--bin-dir", default=os.environ.get("PREPARE_WASM_OUTPUT_DIR", ""))
    ap.add_argument("--tokenizer-dir", default=os.environ.get("PREPARE_WASM_TOKENIZER_DIR", ""))
    ap.add_argument("--public-data-dir", default=os.path.join(os.getcwd(), "public", "data"))
    ap.add_argument("--vocab-size", type=int, default=DEFAULT_VOCAB_SIZE, help="full vocabulary, specials included")
    ap.add_argument("--train-shards", type=int, default=_env_int("PREPARE_WASM_TRAIN_SHARDS", 0, 0))
    ap.add_argument("--train-max-chars", type=int, default=_env_int("PREPARE_WASM_TRAIN_MAX_CHARS", 1_000_000_000, 1))
    ap.add_argument("--train-doc-cap", type=int, default=_env_int("PREPARE_WASM_TRAIN_DOC_CAP", 10_000, 1))
    ap.add_argument("--tokenize-shards", type=int, default=_env_int("PREPARE_WASM_TOKENIZE_SHARDS", 0, 0))
    ap.add_argument("--no-parity", action="store_true", help="skip the parity mirror and manifest")
    ap.add_argument("--workers", type=int, default=os.cpu_count() or 1, help="encoding threads")
    args = ap.parse_args(argv)
    text_dir = args.text_dir or os.path.join(args.cache_dir, "text")
    bin_dir = args.bin_dir or os.path.join(args.cache_dir, "bin")
    tok_dir = args.tokenizer_dir or os.path.join(args.cache_dir, "tokenizer")
    if not os.path.isdir(text_dir):
        print(f"text directory {text_dir} not found: add extracted shard_*.txt files there first", file=sys.stderr)
        return 1
    files = sorted(f for f in os.listdir(text_dir) if f.endswith(".txt"))
    train_files = [f for f in files if VAL_SHARD_MARK not in f]
    val_files = [f for f in files if VAL_SHARD_MARK in f]
    print(f"found {len(train_files)} training shards and {len(val_files)} validation shards")
    use = train_files[:args.train_shards] if args.train_shards > 0 else train_files
    docs, chars = collect_training_corpus(text_dir, use, args.train_max_chars, args.train_doc_cap)
    if not docs:
        raise SystemExit("no training documents collected")
    print(f"training on {len(docs):,} documents ({chars:,} characters)")
    t0 = time.time()
    tok = BPETokenizer()
    if args.workers > 1:  # the chunk split of the training corpus runs on threads
        with tok.pool(args.workers) as count_pool:
            tok.train(docs, args.vocab_size - len(SPECIAL_TOKENS), pool=count_pool)
    else:
        tok.train(docs, args.vocab_size - len(SPECIAL_TOKENS))
    print(f"tokenizer trained in {time.time() - t0:.1f}s (vocab={tok.vocab_size()}, merges={tok.num_merges()})")
    sample = "Hello world! Numbers: 123. Unicode: 你好"
    ids = tok.encode(sample)
    print(f"input:   {sample}\nencoded: {list(map(int, ids))}\ndecoded: {tok.decode(ids)}")
    tok.save(tok_dir)
    print(f"tokenizer bundle saved to {tok_dir}")
    os.makedirs(bin_dir, exist_ok=True)
    pool = tok.pool(args.workers) if args.workers > 1 else None
    try:
        for name in files[:args.tokenize_shards] if args.tokenize_shards > 0 else files:
            t1 = time.time()
            nd, nt = tokenize_shard(tok, os.path.join(text_dir, name), os.path.join(bin_dir, name[:-4] + ".bin"),
                                    pool=pool)
            print(f"  {name}: {nd:,} docs / {nt:,} tokens in {time.time() - t1:.1f}s")
    finally:
        if pool is not None:
            pool.shutdown()
    if not args.no_parity:
        os.makedirs(args.public_data_dir, exist_ok=True)
        m = sync_parity_artifacts(args.cache_dir, bin_dir, tok_dir, args.public_data_dir)
        print(f"parity manifest written to {m}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
