import numpy as np
import pytest

from bitresearch_b200.config import preset
from bitresearch_b200.data.loader import BestFitDocumentBatcher, TokenDataLoader
from bitresearch_b200.data.pipeline import make_batch_source
from bitresearch_b200.data.synthetic import UniformBOSStream, ZipfDocumentSource, bos_id, make_token_bytes


def test_token_loader_wraps_and_targets_shift():
    tl = TokenDataLoader(np.arange(10, dtype=np.int32))
    x, y = tl.next_batch(2, 3)
    assert x.tolist() == [[0, 1, 2], [3, 4, 5]] and y.tolist() == [[1, 2, 3], [4, 5, 6]]
    x, y = tl.next_batch(2, 3)
    assert x.tolist() == [[6, 7, 8], [9, 0, 1]] and y.tolist() == [[7, 8, 9], [0, 1, 2]]
    assert tl.epochs == 1
    val = TokenDataLoader(np.arange(100, dtype=np.int32)).val_split(0.1)
    assert val.tolist() == list(range(90, 100))
    x, y = TokenDataLoader.batch_from_array(np.arange(5, dtype=np.int32), 1, 4, 3)
    assert x.tolist() == [[3, 4, 0, 1]] and y.tolist() == [[4, 0, 1, 2]]


def test_best_fit_packing_reference_semantics():
    docs = [[1] * 5, [2] * 3, [3] * 9, [4] * 2, [5] * 4]
    b = BestFitDocumentBatcher(docs, bos_id=0, buffer_size=3)
    rows = b.pack_rows(2, 7)  # capacity 8
    # buffer [6,4,10] -> 6 fits (largest <=8) -> rem 2 -> refill [4,10,3] nothing fits -> crop shortest (3 -> [0,4])
    assert rows[0].tolist() == [0, 1, 1, 1, 1, 1, 0, 4]
    assert rows[1, 0] == 0  # every row starts at a BOS


@pytest.mark.parametrize("buffer_size", [1, 4, 50])
def test_native_packer_matches_python(buffer_size):
    nd = pytest.importorskip("bitresearch_b200._native_data")
    rng = np.random.default_rng(0)
    docs = [rng.integers(0, 50, size=int(rng.integers(1, 40)), dtype=np.int32) for _ in range(300)]
    offs = np.zeros(len(docs) + 1, np.int64)
    np.cumsum([len(d) for d in docs], out=offs[1:])
    toks = np.concatenate(docs)
    p = nd.corpus_packer(63, buffer_size, toks, offs, False)
    py = BestFitDocumentBatcher(docs, bos_id=63, buffer_size=buffer_size)
    for _ in range(5):
        rows = np.empty((4, 33), np.int32)
        ep = nd.pack_rows(p, rows, 4, 32)
        assert np.array_equal(rows, py.pack_rows(4, 32))
        assert ep == py.epoch


def test_zipf_sources_are_seeded_and_bos_packed():
    nd = pytest.importorskip("bitresearch_b200._native_data")
    V = 512
    a = nd.zipf_packer(V, 1.1, 64.0, 7, 100, 0)
    b = nd.zipf_packer(V, 1.1, 64.0, 7, 100, 0)
    ra, rb = np.empty((8, 129), np.int32), np.empty((8, 129), np.int32)
    nd.pack_rows(a, ra, 8, 128)
    nd.pack_rows(b, rb, 8, 128)
    assert np.array_equal(ra, rb)
    assert (ra[:, 0] == V - 1).all() and ra.max() < V and ra.min() >= 0
    frac_bos = (ra == V - 1).mean()
    assert 0.005 < frac_bos < 0.1  # about 1/(mean_len+1) BOS density
    counts = np.bincount(ra[ra != V - 1].ravel(), minlength=V)
    assert counts.max() > 20 * np.median(counts[counts > 0])  # heavy head of a Zipf law
    py = ZipfDocumentSource(V, 1.1, 64, seed=1).documents(2000)
    assert 50 < np.mean([len(d) for d in py]) < 80


def test_uniform_stream_and_token_bytes():
    s = UniformBOSStream(512, 64, seed=0)
    t = s.take(256)
    assert (t[::64] == bos_id(512)).all() and t.max() < 512
    tb = make_token_bytes(512, 4)
    assert tb[bos_id(512)] == 0 and tb.min() == 0 and tb.max() == 4 and (tb[:-1] >= 1).all()


def test_pipeline_ranks_get_distinct_streams():
    cfg = preset("tiny-cpu")
    a = make_batch_source(cfg, "train", 0, 2).next(2, 16)[0]
    b = make_batch_source(cfg, "train", 1, 2).next(2, 16)[0]
    v = make_batch_source(cfg, "val", 0, 2).next(2, 16)[0]
    assert not np.array_equal(a, b) and not np.array_equal(a, v)


@pytest.mark.parametrize("data", ["zipf", "markov"])
def test_ranks_and_splits_sample_one_distribution(data):
    pytest.importorskip("bitresearch_b200._native_data")
    from bitresearch_b200.config import apply_overrides
    cfg = apply_overrides(preset("d512"), [f"data={data}"])
    tops, firsts = [], []
    for split, rank in [("train", 0), ("train", 1), ("val", 0)]:
        x, _ = make_batch_source(cfg, split, rank, 2).next(16, 2048)
        ids, c = np.unique(x, return_counts=True)
        tops.append(set(ids[np.argsort(-c)[:3]].tolist()))
        firsts.append(x[:, :64].copy())
    assert tops[0] == tops[1] == tops[2]  # the same frequent ids everywhere
    assert not np.array_equal(firsts[0], firsts[1]) and not np.array_equal(firsts[0], firsts[2])


def _pairs(rows, bos, order):
    succ = {}
    for r in rows:
        for t in range(order, len(r)):
            ctx = tuple(r[t - order:t])
            if r[t] == bos or any(c == bos for c in ctx[-1:]):
                continue
            if order == 2 and ctx[0] == bos:
                continue
            succ.setdefault(ctx, set()).add(int(r[t]))
    return succ


@pytest.mark.parametrize("p1,p2,order", [(1.0, 0.0, 1), (0.0, 1.0, 2)])
def test_markov_successor_tables(p1, p2, order):
    nd = pytest.importorskip("bitresearch_b200._native_data")
    V, K = 256, 3
    p = nd.markov_packer(V, 1.1, 128.0, 5, 77, p1, p2, K, 100, 0)
    rows = np.empty((32, 513), np.int32)
    nd.pack_rows(p, rows, 32, 512)
    succ = _pairs(rows, V - 1, order)
    assert max(len(s) for s in succ.values()) <= K
    assert sum(len(s) > 1 for s in succ.values()) > 10  # several successors are actually used
    # same table seed -> same successors from a different stream
    q = nd.markov_packer(V, 1.1, 128.0, 6, 77, p1, p2, K, 100, 0)
    rows2 = np.empty((32, 513), np.int32)
    nd.pack_rows(q, rows2, 32, 512)
    both = _pairs(rows2, V - 1, order)
    shared = [c for c in both if c in succ]
    assert shared and all(len(succ[c] | both[c]) <= K for c in shared)


def test_markov_nll_matches_sampled_frequencies():
    nd = pytest.importorskip("bitresearch_b200._native_data")
    V, K = 8192, 4
    p = nd.markov_packer(V, 1.1, 4096.0, 1, 2, 1.0, 0.0, K, 100, 0)
    rows = np.empty((64, 4097), np.int32)
    nd.pack_rows(p, rows, 64, 4096)
    nll = nd.markov_nll(p, rows, 64, 4096)
    keep = rows[:, 1:] != V - 1
    assert nll[~keep].sum() == 0 and np.isfinite(nll).all() and (nll[keep] > 0).all()
    w = 2.0 ** -np.arange(K)
    w /= w.sum()
    # pure order-1 chain: at most the branch entropy (two branches of a context may name the same id)
    assert nll[keep].mean() < -(w * np.log(w)).sum() + 0.1
    # exp(-nll) of a transition is its probability: compare with sampled frequencies of frequent contexts
    prev, nxt, q = rows[:, :-1].ravel(), rows[:, 1:].ravel(), np.exp(-nll.ravel())
    inner = (prev != V - 1) & (nxt != V - 1)
    ids, counts = np.unique(prev[inner], return_counts=True)
    checked = 0
    for c in ids[np.argsort(-counts)[:5]]:
        sel = inner & (prev == c)
        n = sel.sum()
        for x in np.unique(nxt[sel]):
            m = sel & (nxt == x)
            assert np.allclose(q[m], q[m][0])  # one probability per transition
            assert abs(m.sum() / n - q[m][0]) < 4 * np.sqrt(0.25 / n) + 1e-3, (c, x)
            checked += 1
        assert abs(sum(q[sel & (nxt == x)][0] for x in np.unique(nxt[sel])) - 1.0) < 1e-9
    assert checked > 10


def test_json_documents_and_tokens_payloads(tmp_path):
    import json
    from bitresearch_b200.config import apply_overrides
    from bitresearch_b200.data.loader import find_manifest, load_json_payload
    rng = np.random.default_rng(0)
    docs = [rng.integers(0, 100, size=int(rng.integers(3, 40))).tolist() for _ in range(50)]
    p = tmp_path / "docs.json"
    p.write_text(json.dumps({"documents": docs}))
    kind, got = load_json_payload(str(p))
    assert kind == "documents" and len(got) == 50 and got[3].tolist() == docs[3]
    assert find_manifest(str(p)) is None  # a payload is not a manifest
    t = tmp_path / "toks.json"
    t.write_text(json.dumps(list(range(300))))
    assert load_json_payload(str(t))[0] == "tokens"
    for prefixed in (False, True):
        d = [[127] + x for x in docs] if prefixed else docs
        p.write_text(json.dumps(d))
        cfg = apply_overrides(preset("tiny-cpu"), ["data=documents", f"data_path={p}", "model.vocab_size=128",
                                                   f"documents_bos_prefixed={str(prefixed).lower()}"])
        src = make_batch_source(cfg, "train", 0, 1)
        x, y = src.next(4, 32)
        assert (x[:, 0] == 127).all()  # every row starts with BOS
        assert np.array_equal(x[:, 1:], y[:, :-1])
        # rows are made of whole (or cropped) training documents: the first one follows the first BOS
        train = docs[:45]
        first = x[0, 1:1 + len(train[0])].tolist()
        assert any(first == dd[:len(first)] for dd in train)
        val = make_batch_source(cfg, "val", 0, 1)
        vx, _ = val.next(1, 16)
        assert vx[0, 0] == 127
    # data=tokens with a .json token list
    cfg = apply_overrides(preset("tiny-cpu"), ["data=tokens", f"data_path={t}"])
    x, y = make_batch_source(cfg, "train", 0, 1).next(2, 8)
    assert x[0].tolist() == list(range(8)) and y[0].tolist() == list(range(1, 9))


def test_prefetcher_hands_a_data_error_to_the_consumer():
    """A failing source must surface in get() instead of leaving the training loop waiting."""
    from queue import Queue

    import torch
    from bitresearch_b200.data.pipeline import PinnedPrefetcher

    class Broken:
        def next(self, b, t):
            raise ValueError("corrupt shard")

    p = PinnedPrefetcher.__new__(PinnedPrefetcher)  # no CUDA here: only the host side is exercised
    p.source, p.batch, p.seq = Broken(), 2, 4
    p.host = [(torch.zeros(2, 4, dtype=torch.int32), torch.zeros(2, 4, dtype=torch.int32))]
    p.free, p.ready, p._stop, p._error = Queue(), Queue(), False, None
    p.free.put(0)
    p._fill()
    with pytest.raises(RuntimeError, match="corrupt shard"):
        p.get()
    # a later call (cleanup, eval) raises as well instead of blocking on the empty queue
    with pytest.raises(RuntimeError, match="corrupt shard"):
        p.get()
    p._error = None  # the queue still holds the sentinel for a consumer that bypasses the flag
    with pytest.raises(RuntimeError):
        p.get()
