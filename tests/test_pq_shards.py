"""Host logic of list-sharded IVF-PQ (no GPU): whole inverted lists are spread
over the ranks by pq.list_owners, and IVFPQIndex.shard_lists_by_list cuts a
global index into the shard each rank uploads."""
import numpy as np
import pytest

from meltan_b200 import pq as mpq
from meltan_b200.pq import IVFPQIndex


def _index(rng, nlist, n):
    assign = rng.integers(0, nlist, n)
    assign[: n // 3] = 0  # one long list
    flat = np.argsort(assign, kind="stable").astype(np.uint32)
    off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=nlist))]).astype(np.int64)
    return off, flat


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_list_owners_cover_and_balance(world):
    rng = np.random.default_rng(world)
    off, _ = _index(rng, 97, 5000)
    sizes = np.diff(off)
    owner = mpq.list_owners(sizes, world)
    assert owner.shape == sizes.shape
    assert owner.min() >= 0 and owner.max() < world
    load = np.bincount(owner, weights=sizes, minlength=world)
    # greedy largest-first: every rank within one list of the lightest
    assert load.max() - load.min() <= sizes.max()
    np.testing.assert_array_equal(owner, mpq.list_owners(sizes, world))  # deterministic


@pytest.mark.parametrize("world", [2, 3])
def test_shard_lists_by_list_partition(world):
    rng = np.random.default_rng(7)
    off, flat = _index(rng, 40, 3000)
    owner = mpq.list_owners(np.diff(off), world)
    seen = []
    for r in range(world):
        soff, sflat, spos = IVFPQIndex.shard_lists_by_list(off, flat, owner == r)
        assert len(soff) == len(off)
        sizes = np.diff(soff)
        np.testing.assert_array_equal(sizes[owner != r], 0)
        np.testing.assert_array_equal(sizes[owner == r], np.diff(off)[owner == r])
        for lst in np.flatnonzero(owner == r):
            ids = sflat[soff[lst]:soff[lst + 1]]
            np.testing.assert_array_equal(ids, flat[off[lst]:off[lst + 1]])  # insertion order
            np.testing.assert_array_equal(spos[soff[lst]:soff[lst + 1]], np.arange(len(ids)))
        seen.append(sflat)
    allids = np.sort(np.concatenate(seen))
    np.testing.assert_array_equal(allids, np.sort(flat))
