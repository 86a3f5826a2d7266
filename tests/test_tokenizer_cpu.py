"""Data preparation: the native BPE trainer against a naive recount trainer, tokenizer round trips,
artifact formats, and prepare -> parity manifest -> trainer on CPU."""
import collections
import json
import os
import random

import numpy as np
import pytest

from bitresearch_b200.data.loader import discover_token_bytes, find_manifest, load_token_data, manifest_artifacts
from bitresearch_b200.data.tokenizer import SPECIAL_TOKENS, BPETokenizer


def _corpus(n_docs=300, seed=0):
    rng = random.Random(seed)
    words = ["the", "quick", "brown", "fox", "jumps", "over", "lazy", "dog", "and", "runs", "away", "from",
             "hunters", "in", "forest", "42", "2024", "ünïcödé", "naïve", "café", "你好", "世界", "it's", "we're"]
    docs = []
    for _ in range(n_docs):
        k = rng.randint(3, 40)
        s = " ".join(rng.choice(words) if rng.random() < 0.6 else
                     "".join(rng.choice("abcdefghijklmnop") for _ in range(rng.randint(2, 9))) for _ in range(k))
        s += rng.choice([".", "!", "?", "...", " :)", "\t(x)"])
        docs.append(s)
    return docs


def _naive_train(tok, texts, vocab_size):
    """Recounts every pair after every merge; ties to the smallest (left, right) pair."""
    counts = tok.chunk_counts(texts)
    words = [list(c.encode("utf-8")) for c in counts]
    freq = list(counts.values())
    merges = []
    while 256 + len(merges) < vocab_size:
        pc = collections.Counter()
        for w, f in zip(words, freq):
            for a, b in zip(w, w[1:]):
                pc[(a, b)] += f
        if not pc:
            break
        best = min(pc.items(), key=lambda kv: (-kv[1], kv[0]))[0]
        nid = 256 + len(merges)
        merges.append(best)
        for i, w in enumerate(words):
            out, j = [], 0
            while j < len(w):
                if j + 1 < len(w) and (w[j], w[j + 1]) == best:
                    out.append(nid)
                    j += 2
                else:
                    out.append(w[j])
                    j += 1
            words[i] = out
    return merges


def test_native_trainer_matches_naive_recount():
    docs = _corpus()
    tok = BPETokenizer().train(docs, 256 + 120)
    assert tok.num_merges() == 120
    assert [tuple(m) for m in tok.merges] == [tuple(m) for m in _naive_train(BPETokenizer(), docs, 256 + 120)]
    # deterministic
    assert BPETokenizer().train(docs, 256 + 120).merges == tok.merges


def test_gpt4_split_pattern():
    tok = BPETokenizer()
    chunks = tok._re.findall("Hello world! Numbers: 123. Unicode: 你好\n\nIt's  done")
    assert chunks == ["Hello", " world", "!", " Numbers", ":", " ", "12", "3", ".", " Unicode", ":", " 你好", "\n\n",
                      "It", "'s", " ", " done"]


def test_encode_decode_round_trip_and_artifacts(tmp_path):
    docs = _corpus()
    tok = BPETokenizer().train(docs, 256 + 200)
    for d in docs[:50] + ["Hello world! Numbers: 123. Unicode: 你好", "unseen wørds ✓ 😀"]:
        ids = tok.encode(d)
        assert ids.dtype == np.int32
        assert tok.decode(ids) == d
        assert ids.max() < tok.vocab_size()
    # merges shorten the text
    assert sum(len(tok.encode(d)) for d in docs) < 0.6 * sum(len(d.encode()) for d in docs)
    tj, tb = tok.save(str(tmp_path))
    meta = json.load(open(tj))
    assert meta["vocabSize"] == 456 and meta["fullVocabSize"] == 460 and meta["numMerges"] == 200
    assert meta["specialTokens"] == SPECIAL_TOKENS and meta["bosTokenId"] == 456
    assert meta["specialTokenIds"]["<|reserved_3|>"] == 459
    table = np.fromfile(tb, dtype="<i4")
    assert table.shape == (460,) and (table[456:] == 0).all() and (table[:256] == 1).all()
    assert all(table[256 + i] == len(tok.vocab_bytes()[256 + i]) for i in range(200))
    back = BPETokenizer.load(tj)
    assert back.merges == tok.merges
    for d in docs[:50]:
        assert np.array_equal(back.encode(d), tok.encode(d))


def test_prepare_manifest_and_trainer(tmp_path):
    from bitresearch_b200.data import prepare
    cache = tmp_path / "cache"
    text = cache / "text"
    text.mkdir(parents=True)
    docs = _corpus(600, seed=1)
    (text / "shard_00000.txt").write_text("\n".join(docs[:500]) + "\n\n")
    (text / "shard_06542.txt").write_text("\n".join(docs[500:]) + "\n")
    public = tmp_path / "public"
    rc = prepare.main(["--cache-dir", str(cache), "--public-data-dir", str(public), "--vocab-size", "512"])
    assert rc == 0
    man = find_manifest(str(public))
    assert man == str(public / "parity" / "manifest.json")
    art = manifest_artifacts(man)
    assert [os.path.basename(b) for b in art["bin"]] == ["shard_00000.bin", "shard_06542.bin"]
    assert art["token_bytes"].endswith(os.path.join("tokenizer", "token_bytes.bin"))
    tok = BPETokenizer.load(art["tokenizer"])
    stream = load_token_data(str(public))
    assert stream.dtype == np.int32
    # every document is BOS + its encoding, in file order
    expect = []
    for d in docs[:500] + docs[500:]:
        expect.append(tok.bos_id)
        expect.extend(tok.encode(d).tolist())
    assert stream.tolist() == expect
    assert (stream == tok.bos_id).sum() == 600
    meta = json.load(open(public / "tokens_meta.json"))
    assert meta["source"] == "shard_00000.bin" and meta["vocabSize"] == 512
    assert discover_token_bytes(str(public)) == art["token_bytes"]
    # the trainer consumes the prepared stream and its token_bytes table
    import torch
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.train import Trainer
    cfg = apply_overrides(preset("tiny-cpu"), ["data=tokens", f"data_path={public}", "log_every=0", "results_tsv="])
    tr = Trainer(cfg, device=torch.device("cpu"), log=lambda m: None)
    tr.initialize()
    assert np.array_equal(tr.token_bytes, np.fromfile(art["token_bytes"], dtype="<i4"))
    loss = float(tr.train_step())
    assert np.isfinite(loss)
    tr.destroy()


def test_pooled_encoding_matches_serial(tmp_path):
    docs = _corpus(400, seed=2)
    tok = BPETokenizer().train(docs, 256 + 150)
    with tok.pool(2) as pool:
        pooled = tok.batch_encode(docs, pool=pool, chunk=16)
    serial = tok.batch_encode(docs)
    assert len(pooled) == len(serial) and all(np.array_equal(a, b) for a, b in zip(pooled, serial))


def test_prepare_with_worker_pool_writes_the_same_shards(tmp_path):
    from bitresearch_b200.data import prepare
    outs = []
    for workers in (1, 2):
        cache = tmp_path / f"cache{workers}"
        (cache / "text").mkdir(parents=True)
        docs = _corpus(300, seed=4)
        (cache / "text" / "shard_00000.txt").write_text("\n".join(docs[:250]) + "\n")
        (cache / "text" / "shard_06542.txt").write_text("\n".join(docs[250:]) + "\n")
        assert prepare.main(["--cache-dir", str(cache), "--vocab-size", "400", "--no-parity",
                             "--workers", str(workers)]) == 0
        outs.append([np.fromfile(cache / "bin" / n, dtype=np.int32) for n in ("shard_00000.bin", "shard_06542.bin")])
    assert all(np.array_equal(a, b) for a, b in zip(*outs))


def test_pooled_chunk_counts_match_serial():
    docs = _corpus(500, seed=6)
    tok = BPETokenizer()
    with tok.pool(2) as pool:
        pooled = tok.chunk_counts(docs, pool=pool, chunk=64)
    serial = tok.chunk_counts(docs)
    assert pooled == serial
    with tok.pool(2) as pool:
        merges = BPETokenizer().train(docs, 256 + 80, pool=pool).merges
    assert merges == BPETokenizer().train(docs, 256 + 80).merges  # merges depend on the counts, not their order


def test_native_split_matches_the_regex():
    import regex
    nd = pytest.importorskip("bitresearch_b200._native_data")
    from bitresearch_b200.data.tokenizer import SPLIT_PATTERN
    BPETokenizer()  # installs the code-point table
    pat = regex.compile(SPLIT_PATTERN)
    rng = random.Random(1)
    alpha = list("abZQsdmtlvreSDMTLVRE0189'\"  \t\n\r\x0b\x0c.,!?-()_#/;:<>") + [
        "  ", "\n\n", " '", "'s", "'LL", "\r\n", "é", "ß", "\u017f", "你", "²", "½", "\u0663", "\u216b", "\xa0", "\x85",
        "\u3000", "\x1c", "\u200b", "\u201c", "\u2014", "\U0001f600", "\u0301", "\u212a", "\x00", "\x7f"]
    for _ in range(20000):
        s = "".join(rng.choice(alpha) for _ in range(rng.randint(0, 24)))
        assert nd.split_text(s) == pat.findall(s), repr(s)
    chars = [chr(c) for c in range(0x20, 0x7F)] + ["\t", "\n", "\x0b", "\x0c", "\r", "\xa0", "\u017f", "\u2028"]
    for x in chars:
        for y in chars:
            for s in (x + y + "a", " " + x + y, x + "'" + y):
                assert nd.split_text(s) == pat.findall(s), repr(s)


def test_native_and_regex_paths_train_and_encode_alike():
    docs = _corpus(300, seed=7)  # mixes ASCII documents and documents with non-ASCII words
    tok = BPETokenizer()
    native = tok.chunk_counts(docs)
    by_regex = collections.Counter()
    for d in docs:
        by_regex.update(tok._re.findall(d))
    assert native == by_regex
    t = BPETokenizer().train(docs, 256 + 100)
    for d in docs[:100]:
        assert np.array_equal(t.encode(d), t._enc.encode_chunks(t._re.findall(d)))
