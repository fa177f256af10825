"""GPU parity of IVF-PQ search and single-list ADC against the oracle's
restatement of _IVFPQIndex.search (coarse BoundedSortedList, residual LUT,
sequential ADC, newest-first merge) and GPUADCSearch.computeDistances:
identical internal ids, bit-equal scores, identical tie order.  Cases follow
Tests/MetalANNSTests/{IVFPQIndexTests,IVFPQGPUTests,GPUADCSearchTests,
BoundedSelectionTests}.swift."""
import numpy as np
import pytest

import bench
import meltan_b200 as mb
import oracle as O

pytestmark = pytest.mark.gpu


def encode_all(v, coarse, codebooks, metric):
    """_IVFPQIndex.add: nearest coarse centroid (strict <) then
    encode(vector:subtracting:) per vector, lists in insertion order."""
    nlist = coarse.shape[0]
    m = codebooks.shape[0]
    codes = np.zeros((len(v), m), np.uint8)
    lists = [[] for _ in range(nlist)]
    for i, x in enumerate(v):
        c = O.nearest_coarse(x, coarse, metric)
        codes[i] = O.pq_encode_subtracting(x, coarse[c], codebooks)
        lists[c].append(i)
    offsets = np.concatenate([[0], np.cumsum([len(x) for x in lists])]).astype(np.int64)
    flat = np.array(sum(lists, []), np.uint32)
    return codes, offsets, flat


def make_index(n, dim, m, nlist, metric, seed, dup=False):
    rng = np.random.default_rng(seed)
    v, q = bench.make_mixture(n, dim, 16, 20, sigma=0.2, seed=seed)
    if dup:
        v = np.repeat(v[: n // 2], 2, axis=0)
    coarse = v[rng.choice(len(v), nlist, replace=False)].copy()
    codebooks = (rng.standard_normal((m, 256, dim // m)) * 0.1).astype(np.float32)
    codes, offsets, flat = encode_all(v, coarse, codebooks, metric)
    return v, q, coarse, codebooks, codes, offsets, flat


def same(got, want):
    np.testing.assert_array_equal(got[2], want[2])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0], want[0])


@pytest.mark.parametrize("metric", [O.L2, O.COSINE, O.IP])
def test_ivfpq_parity(ctx, metric):
    v, q, coarse, cb, codes, off, flat = make_index(3000, 32, 8, 16, metric, seed=11)
    ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (off, flat), metric=mb.Metric(metric))
    for nprobe in (1, 3, 8, 16, 40):
        for k in (1, 10, 57):
            same(ix.search_arrays(q, k, nprobe),
                 O.ivfpq_search(coarse, cb, codes, off, flat, q, k, nprobe, metric))
    ix.close()


def test_ivfpq_duplicates_merge_newest_first(ctx):
    """BoundedSelectionTests.ivfpqMergeTieOrderPinned (:281-317): duplicate
    vectors a_i, b_i (b inserted after a) come back b_i before a_i."""
    v, q, coarse, cb, codes, off, flat = make_index(2000, 16, 4, 4, O.L2, seed=3, dup=True)
    ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (off, flat))
    got = ix.search_arrays(v[:5], 6, 4)
    want = O.ivfpq_search(coarse, cb, codes, off, flat, v[:5], 6, 4, O.L2)
    same(got, want)
    for r in range(5):
        ids = got[1][r].tolist()
        for a in range(0, 6, 2):
            assert got[0][r, a] == got[0][r, a + 1]
            assert ids[a] == ids[a + 1] + 1
    # massive ties: every code identical -> the order is pure insertion order
    codes0 = np.zeros_like(codes)
    ix0 = mb.IVFPQIndex(ctx, coarse, cb, codes0, (off, flat))
    for k in (1, 5, 37, 256):
        same(ix0.search_arrays(q[:3], k, 4),
             O.ivfpq_search(coarse, cb, codes0, off, flat, q[:3], k, 4, O.L2))
    ix.close()
    ix0.close()


def test_ivfpq_sizes_and_empty_lists(ctx):
    v, q, coarse, cb, codes, off, flat = make_index(5000, 64, 16, 32, O.L2, seed=5)
    far = (np.ones((4, 64), np.float32) * 40)
    coarse2 = np.concatenate([coarse, far])
    codes2, off2, flat2 = encode_all(v, coarse2, cb, O.L2)
    assert (np.diff(off2) == 0).any()
    ix = mb.IVFPQIndex(ctx, coarse2, cb, codes2, (off2, flat2))
    for nq in (1, 7, 20):
        same(ix.search_arrays(q[:nq], 10, 36),
             O.ivfpq_search(coarse2, cb, codes2, off2, flat2, q[:nq], 10, 36, O.L2))
    assert ix.search_arrays(q[:2, :63], 10, 4)[2].tolist() == [0, 0]  # wrong width -> []
    assert ix.search(q[0], 0, 4) == []
    ix.close()


def test_gpu_adc_matches_cpu_adc(ctx):
    """GPUADCSearchTests.swift:10-33 (GPU vs CPU ADC) -- here bit-equal."""
    rng = np.random.default_rng(9)
    cb = rng.standard_normal((16, 256, 8)).astype(np.float32)
    query = rng.standard_normal(128).astype(np.float32)
    codes = rng.integers(0, 256, (5000, 16)).astype(np.uint8)
    got = mb.GPUADCSearch.compute_distances(ctx, query, cb, codes)
    want = O.pq_adc(O.pq_lut(query, cb, O.L2), codes)
    np.testing.assert_array_equal(got, want)
    assert mb.GPUADCSearch.compute_distances(ctx, query, cb, codes[:0]).shape == (0,)


def test_gpu_adc_rejects_out_of_range_codes(ctx):
    """GPUADCSearchTests: codes >= Ks are rejected with searchFailed."""
    rng = np.random.default_rng(1)
    cb = rng.standard_normal((4, 16, 2)).astype(np.float32)
    codes = np.array([[1, 2, 3, 20]], np.uint8)
    with pytest.raises(mb.SearchFailed):
        mb.GPUADCSearch.compute_distances(ctx, rng.standard_normal(8).astype(np.float32), cb, codes)


@pytest.mark.slow
def test_ivfpq_large(ctx):
    """200k x 128, nlist 256, m = 16 (scaled-down C4) against the oracle."""
    v, q = bench.make_mixture(200_000, 128, 256, 12, seed=4)
    coarse, cb, codes, off, flat = bench.train_ivfpq(v, 256, 16)
    ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (off, flat))
    same(ix.search_arrays(q, 10, 32), O.ivfpq_search(coarse, cb, codes, off, flat, q, 10, 32, O.L2))
    ix.close()


@pytest.mark.parametrize("metric", [O.L2, O.COSINE, O.IP])
def test_gpu_encode_matches_reference_encode(ctx, metric):
    """IVFPQIndex.add's encoding on the device: coarse assignment
    (nearestCoarseCentroid) and residual codes (encode(vector:subtracting:))
    equal the oracle's restatement for every vector, including tied codewords
    (duplicated codebook rows: the first index wins)."""
    rng = np.random.default_rng(21)
    n, dim, m = 3000, 64, 8
    v = rng.standard_normal((n, dim), dtype=np.float32)
    coarse = rng.standard_normal((24, dim), dtype=np.float32)
    cb = rng.standard_normal((m, 256, dim // m), dtype=np.float32) * np.float32(0.5)
    cb[:, 200:] = cb[:, 100:156]  # exact duplicates
    codes, assign = mb.pq_encode(ctx, v, coarse, cb, mb.Metric(metric))
    for i in range(0, n, 7):
        a = O.nearest_coarse(v[i], coarse, metric)
        assert assign[i] == a
        np.testing.assert_array_equal(codes[i], O.pq_encode_subtracting(v[i], coarse[a], cb))


def test_gpu_encode_small_codebooks_and_scalar_subspaces(ctx):
    rng = np.random.default_rng(22)
    v = rng.standard_normal((777, 12), dtype=np.float32)
    coarse = v[:5].copy()
    cb = rng.standard_normal((12, 16, 1), dtype=np.float32)  # ks 16, sub 1
    codes, assign = mb.pq_encode(ctx, v, coarse, cb)
    for i in range(777):
        a = O.nearest_coarse(v[i], coarse, O.L2)
        assert assign[i] == a
        np.testing.assert_array_equal(codes[i], O.pq_encode_subtracting(v[i], coarse[a], cb))


@pytest.mark.parametrize("shards", [2, 3])
def test_row_sharded_ivfpq_equals_unsharded(ctx, shards):
    """IVF-PQ over row shards (each with its rows' list entries and their
    global list positions): the shards' (score, sequence) 2k-blocks, merged
    and resolved, equal the oracle's _IVFPQIndex.search on the whole index --
    ties included (duplicate codes make equal scores that newest-first
    ordering decides)."""
    import torch
    from meltan_b200 import pq as mpq
    rng = np.random.default_rng(33)
    n, dim, m, nlist = 6000, 32, 8, 24
    v = rng.standard_normal((n, dim), dtype=np.float32)
    coarse = v[rng.choice(n, nlist, replace=False)].copy()
    cb = rng.standard_normal((m, 256, dim // m), dtype=np.float32)
    codes, assign = mb.pq_encode(ctx, v, coarse, cb)
    codes[4000:4100] = codes[10]  # equal scores across shards
    flat = np.argsort(assign, kind="stable").astype(np.uint32)
    off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=nlist))]).astype(np.int64)
    q = rng.standard_normal((7, dim), dtype=np.float32)
    ws = mb.Workspace(ctx)
    dq = torch.from_numpy(q).cuda()
    for k, nprobe in ((10, 4), (25, 24)):
        words = mpq.partial_words(len(q), k)
        blocks = torch.empty((shards, words), dtype=torch.int32, device="cuda")
        idx = []
        for s_ in range(shards):
            r0, r1 = mb.row_shard(n, shards, s_)
            soff, sflat, spos = mb.IVFPQIndex.shard_lists(off, flat, r0, r1)
            ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (soff, sflat), list_positions=spos)
            ix.search_partial_device(ws, dq.data_ptr(), len(q), k, nprobe, blocks[s_].data_ptr())
            idx.append(ix)
        kout = min(k, 256)
        od = torch.empty((len(q), kout), dtype=torch.float32, device="cuda")
        oi = torch.empty((len(q), kout), dtype=torch.int32, device="cuda")
        oc = torch.empty((len(q),), dtype=torch.int32, device="cuda")
        mpq.resolve_device(ctx, ws, blocks.data_ptr(), shards, words, len(q), k, od.data_ptr(),
                           oi.data_ptr(), oc.data_ptr())
        ws.check()
        want = O.ivfpq_search(coarse, cb, codes, off, flat, q, k, nprobe, O.L2)
        np.testing.assert_array_equal(oc.cpu().numpy(), want[2])
        np.testing.assert_array_equal(oi.cpu().numpy().view(np.uint32), want[1])
        np.testing.assert_array_equal(od.cpu().numpy(), want[0])
        for ix in idx:
            ix.close()
    ws.close()


@pytest.mark.parametrize("shards", [2, 3])
def test_list_sharded_ivfpq_equals_unsharded(ctx, shards):
    """IVF-PQ over list shards (whole inverted lists per shard, spread by
    pq.list_owners): each shard builds tables only for the probed lists it
    holds, and its (score, sequence) 2k-blocks, merged and resolved, equal the
    oracle's _IVFPQIndex.search on the whole index -- ties included."""
    import torch
    from meltan_b200 import pq as mpq
    rng = np.random.default_rng(34)
    n, dim, m, nlist = 6000, 32, 8, 24
    v = rng.standard_normal((n, dim), dtype=np.float32)
    coarse = v[rng.choice(n, nlist, replace=False)].copy()
    cb = rng.standard_normal((m, 256, dim // m), dtype=np.float32)
    codes, assign = mb.pq_encode(ctx, v, coarse, cb)
    codes[4000:4100] = codes[10]  # equal scores in different lists and shards
    flat = np.argsort(assign, kind="stable").astype(np.uint32)
    off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=nlist))]).astype(np.int64)
    owner = mpq.list_owners(np.diff(off), shards)
    q = rng.standard_normal((70, dim), dtype=np.float32)  # the small-corpus coarse step too
    ws = mb.Workspace(ctx)
    dq = torch.from_numpy(q).cuda()
    for k, nprobe in ((10, 4), (25, 24), (3, 1)):
        words = mpq.partial_words(len(q), k)
        blocks = torch.empty((shards, words), dtype=torch.int32, device="cuda")
        idx = []
        for s_ in range(shards):
            soff, sflat, spos = mb.IVFPQIndex.shard_lists_by_list(off, flat, owner == s_)
            ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (soff, sflat), list_positions=spos)
            ix.search_partial_device(ws, dq.data_ptr(), len(q), k, nprobe, blocks[s_].data_ptr())
            idx.append(ix)
        kout = min(k, 256)
        od = torch.empty((len(q), kout), dtype=torch.float32, device="cuda")
        oi = torch.empty((len(q), kout), dtype=torch.int32, device="cuda")
        oc = torch.empty((len(q),), dtype=torch.int32, device="cuda")
        mpq.resolve_device(ctx, ws, blocks.data_ptr(), shards, words, len(q), k, od.data_ptr(),
                           oi.data_ptr(), oc.data_ptr())
        ws.check()
        want = O.ivfpq_search(coarse, cb, codes, off, flat, q, k, nprobe, O.L2)
        np.testing.assert_array_equal(oc.cpu().numpy(), want[2])
        np.testing.assert_array_equal(oi.cpu().numpy().view(np.uint32), want[1])
        np.testing.assert_array_equal(od.cpu().numpy(), want[0])
        for ix in idx:
            ix.close()
    ws.close()


def test_ivfpq_list_longer_than_2_pow_20(ctx):
    """One inverted list of 1.1M entries (beyond 2^20), searched at nprobe 1
    and 2 against the oracle; positions that cannot fit the 32-bit insertion
    sequence at a given nprobe fail with searchFailed instead of merging
    wrongly."""
    rng = np.random.default_rng(31)
    n, dim, m = 1_100_000, 8, 4
    coarse = np.stack([np.zeros(dim, np.float32), np.full(dim, 100, np.float32)])
    cb = (rng.standard_normal((m, 256, dim // m)) * 0.5).astype(np.float32)
    codes = rng.integers(0, 256, (n, m)).astype(np.uint8)
    codes[::7] = codes[3]  # many equal scores: the tie order spans the whole list
    offsets = np.array([0, n - 3, n], np.int64)
    lists = np.arange(n, dtype=np.uint32)
    q = (rng.standard_normal((3, dim)) * 0.3).astype(np.float32)
    ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (offsets, lists))
    for nprobe in (1, 2):
        same(ix.search_arrays(q, 50, nprobe),
             O.ivfpq_search(coarse, cb, codes, offsets, lists, q, 50, nprobe, O.L2))
    ix.close()
    # a shard whose entries report positions up to 2^29 + 2: fine at nprobe 4
    # (positions below 2^30), rejected at nprobe 8 (below 2^29)
    coarse8 = (rng.standard_normal((8, dim)) * 0.1).astype(np.float32)
    small = np.array([0, 3, 6, 6, 6, 6, 6, 6, 6], np.int64)
    pos = np.array([0, 1, (1 << 29) + 2, 0, 1, 2], np.uint32)
    ixs = mb.IVFPQIndex(ctx, coarse8, cb, codes[:6], (small, np.arange(6, dtype=np.uint32)),
                        list_positions=pos)
    # a plain search of such a shard is the search of its own entries (the
    # positions keep their relative order within each list)
    lists6 = np.arange(6, dtype=np.uint32)
    for nprobe in (1, 4):
        same(ixs.search_arrays(q, 5, nprobe),
             O.ivfpq_search(coarse8, cb, codes[:6], small, lists6, q, 5, nprobe, O.L2))
    with pytest.raises(mb.SearchFailed):
        ixs.search_arrays(q, 5, 8)
    ixs.close()
    with pytest.raises(mb.ConstructionFailed):  # positions must ascend within a list
        mb.IVFPQIndex(ctx, coarse8, cb, codes[:6], (small, lists6),
                      list_positions=np.array([0, 5, 5, 0, 1, 2], np.uint32))


@pytest.mark.parametrize("metric", [O.L2, O.COSINE, O.IP])
@pytest.mark.parametrize("dim", [64, 128])
def test_ivfpq_grouped_batches(ctx, metric, dim):
    """Batches of >= 16 queries with m = 16 and k <= 16 run the grouped ADC
    (the queries probing one list share its code reads, tables built 1, 2 or
    4 wide by the tile's query count).  Queries drawn near a few centroids
    make hot lists (many tiles per list), duplicate codes make ties; every
    query equals the oracle, ids, scores and tie order."""
    rng = np.random.default_rng(dim + metric)
    n, m, nlist = 12000, 16, 40
    v, _ = bench.make_mixture(n, dim, 30, 1, sigma=0.3, seed=dim)
    coarse = v[rng.choice(n, nlist, replace=False)].copy()
    cb = (rng.standard_normal((m, 256, dim // m)) * 0.2).astype(np.float32)
    codes, offsets, flat = encode_all(v, coarse, cb, metric)
    codes[flat[: len(flat) // 3: 5]] = codes[flat[0]]  # many equal scores
    hot = coarse[:3][rng.integers(0, 3, 300)] + np.float32(0.05) * rng.standard_normal(
        (300, dim), dtype=np.float32)
    ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (offsets, flat), metric=mb.Metric(metric))
    for nq, q in ((16, hot[:16]), (41, hot[:41]), (300, hot)):
        for k, nprobe in ((1, 1), (5, 3), (10, 8), (16, nlist)):
            same(ix.search_arrays(q, k, nprobe),
                 O.ivfpq_search(coarse, cb, codes, offsets, flat, q, k, nprobe, metric))
    ix.close()


@pytest.mark.parametrize("shards", [2, 3])
def test_list_sharded_grouped_ivfpq(ctx, shards):
    """List shards through the grouped ADC (m = 16, 64 queries): the shards'
    blocks, merged and resolved, equal the oracle on the whole index."""
    import torch
    from meltan_b200 import pq as mpq
    rng = np.random.default_rng(35)
    n, dim, m, nlist = 8000, 64, 16, 30
    v = rng.standard_normal((n, dim), dtype=np.float32)
    coarse = v[rng.choice(n, nlist, replace=False)].copy()
    cb = rng.standard_normal((m, 256, dim // m), dtype=np.float32)
    codes, assign = mb.pq_encode(ctx, v, coarse, cb)
    codes[5000:5200] = codes[10]
    flat = np.argsort(assign, kind="stable").astype(np.uint32)
    off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=nlist))]).astype(np.int64)
    owner = mpq.list_owners(np.diff(off), shards)
    q = rng.standard_normal((64, dim), dtype=np.float32)
    ws = mb.Workspace(ctx)
    dq = torch.from_numpy(q).cuda()
    for k, nprobe in ((10, 4), (16, 30)):
        words = mpq.partial_words(len(q), k)
        blocks = torch.empty((shards, words), dtype=torch.int32, device="cuda")
        idx = []
        for s_ in range(shards):
            soff, sflat, spos = mb.IVFPQIndex.shard_lists_by_list(off, flat, owner == s_)
            ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (soff, sflat), list_positions=spos)
            ix.search_partial_device(ws, dq.data_ptr(), len(q), k, nprobe, blocks[s_].data_ptr())
            idx.append(ix)
        od = torch.empty((len(q), k), dtype=torch.float32, device="cuda")
        oi = torch.empty((len(q), k), dtype=torch.int32, device="cuda")
        oc = torch.empty((len(q),), dtype=torch.int32, device="cuda")
        mpq.resolve_device(ctx, ws, blocks.data_ptr(), shards, words, len(q), k, od.data_ptr(),
                           oi.data_ptr(), oc.data_ptr())
        ws.check()
        want = O.ivfpq_search(coarse, cb, codes, off, flat, q, k, nprobe, O.L2)
        np.testing.assert_array_equal(oc.cpu().numpy(), want[2])
        np.testing.assert_array_equal(oi.cpu().numpy().view(np.uint32), want[1])
        np.testing.assert_array_equal(od.cpu().numpy(), want[0])
        for ix in idx:
            ix.close()
    ws.close()


@pytest.mark.parametrize("metric", [O.L2, O.COSINE, O.IP])
def test_ivfpq_k_above_256(ctx, metric):
    """k above 256: BoundedSortedList(capacity: k) has no cap beyond k
    (IVFPQIndex.swift:197), so results are k wide; every probed entry's key
    is sorted per query on the device.  k below, at and above the candidate
    count, ties from duplicated codes, and single queries."""
    v, q, coarse, cb, codes, off, flat = make_index(6000, 32, 8, 16, metric, seed=41)
    ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (off, flat), metric=mb.Metric(metric))
    for nprobe in (1, 4, 16):
        for k in (257, 700, 6000, 9000):
            same(ix.search_arrays(q, k, nprobe),
                 O.ivfpq_search(coarse, cb, codes, off, flat, q, k, nprobe, metric))
    same(ix.search_arrays(q[:1], 300, 3),
         O.ivfpq_search(coarse, cb, codes, off, flat, q[:1], 300, 3, metric))
    ix.close()


def test_ivfpq_k_above_256_ties(ctx):
    """Heavy ties with k above 256: duplicated vectors (newest first among
    equal scores) and every code identical (pure insertion order, with the
    equal-score entries past the k-th rejected)."""
    v, q, coarse, cb, codes, off, flat = make_index(3000, 16, 4, 4, O.L2, seed=43, dup=True)
    ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (off, flat))
    for k in (300, 1001, 2999):
        same(ix.search_arrays(v[:4], k, 4),
             O.ivfpq_search(coarse, cb, codes, off, flat, v[:4], k, 4, O.L2))
    codes0 = np.zeros_like(codes)
    ix0 = mb.IVFPQIndex(ctx, coarse, cb, codes0, (off, flat))
    for k in (257, 512, 1500, 3000, 4000):
        for nprobe in (1, 2, 4):
            same(ix0.search_arrays(q[:3], k, nprobe),
                 O.ivfpq_search(coarse, cb, codes0, off, flat, q[:3], k, nprobe, O.L2))
    ix.close()
    ix0.close()
