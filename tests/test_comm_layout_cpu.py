"""Host-side layout of the NVLink data-parallel path: gradient buckets in backward order, the flat
buffer layout, parameter ownership and chunk tables (pure functions, no GPU)."""
import numpy as np
import pytest

from bitresearch_b200.config import preset
from bitresearch_b200.models.gpt import GPT
from bitresearch_b200.parallel.comm import (ALIGN, assign_owners, bucket_order, chunk_ranges, flat_layout,
                                             interleave_by_owner)


def _specs(name="d512", **model):
    cfg = preset(name).model
    for k, v in model.items():
        setattr(cfg, k, v)
    return GPT(cfg, device="meta").specs, cfg


def test_buckets_follow_backward_completion():
    specs, cfg = _specs()
    buckets = bucket_order(specs, cfg.n_layer)
    names = [n for n, _, _ in specs]
    flat = [n for b in buckets for n in b]
    assert sorted(flat) == sorted(names) and len(flat) == len(set(flat))  # every parameter exactly once
    assert buckets[0] == ["lmHead"] and set(buckets[-1]) == {"wte", "residLambdas", "x0Lambdas"}
    layer_of = [int(b[0][5:].split("_")[0]) for b in buckets[1:-1]]
    assert layer_of == list(reversed(range(cfg.n_layer)))  # the last layer's gradients are final first
    for i, b in zip(layer_of, buckets[1:-1]):
        assert all(n.startswith(f"layer{i}_") or n == f"ve_{i}" for n in b)


def test_flat_layout_is_aligned_disjoint_and_bucket_contiguous():
    specs, cfg = _specs()
    layout, ranges, groups, total = flat_layout(specs, cfg.n_layer)
    spans = sorted((off, off + numel) for off, numel, _ in layout.values())
    assert all(off % ALIGN == 0 for off, _ in spans)
    assert all(a_end <= b_start for (_, a_end), (b_start, _) in zip(spans, spans[1:]))
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    assert all(r1[1] == r2[0] for r1, r2 in zip(ranges, ranges[1:]))
    for (lo, hi), grp in zip(ranges, groups):
        for n in grp:
            off, numel, shape = layout[n]
            assert lo <= off and off + numel <= hi and numel == int(np.prod(shape))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_owner_assignment_is_complete_deterministic_and_balanced(world):
    specs, _ = _specs()
    own = assign_owners(specs, world)
    assert set(own) == {n for n, _, _ in specs} and set(own.values()) == set(range(world))
    assert own == assign_owners(list(reversed(specs)), world)  # the same on every rank, whatever the order
    counts = np.bincount([own[n] for n, _, _ in specs], minlength=world)
    assert counts.min() >= 1
    # element load per rank: greedy LPT stays within the largest single tensor of the mean
    sizes = {n: int(np.prod(s)) for n, s, _ in specs}
    load = np.zeros(world)
    for n, r in own.items():
        load[r] += sizes[n]
    assert load.max() - load.mean() <= max(sizes.values())


def test_chunk_ranges_cover_exactly():
    for numel in (1, 1000, 65536, 65537, 300_001):
        ch = chunk_ranges(4096, numel, start_in_param=7, size=65536)
        assert ch[0][0] == 4096 and sum(ln for _, ln, _ in ch) == numel
        assert all(0 < ln <= 65536 for _, ln, _ in ch)
        assert all(a[0] + a[1] == b[0] and a[2] + a[1] == b[2] for a, b in zip(ch, ch[1:]))
        assert ch[0][2] == 7


@pytest.mark.parametrize("world", [2, 4, 8])
def test_push_rows_interleave_owners_from_the_next_rank(world):
    """Every row kept once, order within an owner kept, each round visits the owners from rank + 1 on
    (this rank's own rows last), so the ranks start on different peers."""
    rows = [(10 * o + i, 1, o, i) for o in range(world) for i in range(3 + o)]  # uneven shares
    for rank in range(world):
        out = interleave_by_owner(rows, rank, world)
        assert sorted(out) == sorted(rows)
        for o in range(world):
            assert [r for r in out if r[2] == o] == [r for r in rows if r[2] == o]
        first = [r[2] for r in out[:world]]
        assert first == [(rank + 1 + k) % world for k in range(world)]
    starts = {interleave_by_owner(rows, rank, world)[0][2] for rank in range(world)}
    assert len(starts) == world
