"""The reference ring algorithm over gloo: correct mean, f16 wire, abort on a silent peer."""
import numpy as np
import pytest
import torch

from dist_utils import run_world


def _ring(rank, world, wire, P):
    from bitresearch_b200.parallel.ring import RingAllReduce
    g = torch.from_numpy(np.random.default_rng(rank).standard_normal(P).astype(np.float32))
    out = RingAllReduce(wire_dtype=wire, timeout_s=20).all_reduce(g, step_id=3)
    return out.numpy()


@pytest.mark.parametrize("world,wire,P", [(2, "fp32", 1000), (3, "fp32", 1001), (4, "fp16", 4099)])
def test_ring_mean(world, wire, P):
    outs = run_world(_ring, world, wire, P)
    expect = np.mean([np.random.default_rng(r).standard_normal(P).astype(np.float32) for r in range(world)], 0)
    tol = 1e-6 if wire == "fp32" else 2e-3
    for o in outs:
        np.testing.assert_allclose(o, expect, atol=tol)
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])  # every rank ends with identical values


def _ring_abort(rank, world):
    import time

    from bitresearch_b200.parallel.ring import RingAllReduce
    if rank == 1:
        time.sleep(4.0)  # never joins this collective (a peer that went silent)
        return "silent"
    out = RingAllReduce(wire_dtype="fp32", timeout_s=1.0).all_reduce(torch.ones(64), 0)
    return out is None


def test_ring_abort_returns_none():
    res = run_world(_ring_abort, 2)
    assert res[0] is True
