"""Host side of the row-sharded search at world_size 2 over gloo (CPU): shard
bounds, global ids through the shard offset, the packed per-rank block and
the single all-gather.  Each rank's list comes from the oracle on its shard;
the gathered lists merged by (distance, id) must equal the unsharded oracle
search (the mergeSorted contract, ParallelFlatScan.swift:288-315)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from meltan_b200 import shard

N, DIM, NQ, K = 3001, 24, 5, 10


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, metric, out_dir):
    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        v = O.lcg_vectors(N, DIM, 5)
        q = O.lcg_vectors(NQ, DIM, 6)
        r0, r1 = shard.row_shard(N, world, rank)
        d, i, c = O.flat_search(v[r0:r1], q, K, metric)
        kout = d.shape[1]
        loc = torch.zeros(shard.packed_words(NQ, kout), dtype=torch.int32)
        bd, bi, bc = shard.block_views(loc, NQ, kout)
        bd.copy_(torch.from_numpy(d))
        ids = i.astype(np.int64)
        ids = np.where(ids == 0xFFFFFFFF, ids, ids + r0)  # global ids, empty slots kept
        bi.copy_(torch.from_numpy(ids.astype(np.uint32).view(np.int32)))
        bc.copy_(torch.from_numpy(c))
        gat = torch.empty((world, loc.numel()), dtype=torch.int32)
        shard.all_gather_blocks(dist, loc, gat)
        np.save(os.path.join(out_dir, f"gathered{rank}.npy"), gat.numpy())
    finally:
        dist.destroy_process_group()


def merge(gathered, nq, kout, k):
    """(distance, id) merge of the per-rank ascending lists."""
    md = np.full((nq, kout), np.inf, np.float32)
    mi = np.full((nq, kout), 0xFFFFFFFF, np.uint32)
    mc = np.zeros(nq, np.int32)
    for qi in range(nq):
        pairs = []
        for blk in gathered:
            bd, bi, bc = shard.block_views(torch.from_numpy(blk), nq, kout)
            for j in range(int(bc[qi])):
                pairs.append((float(bd[qi, j]), int(bi[qi, j]) & 0xFFFFFFFF))
        pairs.sort()
        pairs = pairs[:min(k, kout)]
        mc[qi] = len(pairs)
        for j, (dd, ii) in enumerate(pairs):
            md[qi, j], mi[qi, j] = dd, ii
    return md, mi, mc


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_two_rank_gather_equals_unsharded(tmp_path, metric):
    import oracle as O

    world = 2
    mp.start_processes(worker, args=(world, free_port(), metric, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    g0 = np.load(tmp_path / "gathered0.npy")
    g1 = np.load(tmp_path / "gathered1.npy")
    np.testing.assert_array_equal(g0, g1)  # every rank sees the same blocks, rank order
    v = O.lcg_vectors(N, DIM, 5)
    q = O.lcg_vectors(NQ, DIM, 6)
    want = O.flat_search(v, q, K, metric)
    got = merge(g0, NQ, want[0].shape[1], K)
    np.testing.assert_array_equal(got[2], want[2])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0], want[0])


def test_row_shard_matches_array_split():
    for n in (0, 1, 7, 64, 1000, 1_000_001):
        for world in (1, 2, 3, 8):
            parts = np.array_split(np.arange(n), world)
            covered = 0
            for r in range(world):
                r0, r1 = shard.row_shard(n, world, r)
                assert r1 - r0 == len(parts[r])
                if len(parts[r]):
                    assert r0 == parts[r][0]
                assert r0 == covered
                covered = r1
            assert covered == n
    with pytest.raises(ValueError):
        shard.row_shard(10, 2, 2)


def test_block_views_layout():
    nq, kout = 3, 4
    blk = torch.arange(shard.packed_words(nq, kout), dtype=torch.int32)
    d, i, c = shard.block_views(blk, nq, kout)
    assert d.shape == (nq, kout) and i.shape == (nq, kout) and c.shape == (nq,)
    assert int(i[0, 0]) == nq * kout and int(c[0]) == 2 * nq * kout
    with pytest.raises(ValueError):
        shard.block_views(blk[:-1], nq, kout)
