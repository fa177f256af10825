"""GPU parity of IVF-flat probe-and-scan against the oracle's restatement of
IVFFlatSearch.scanProbedLists (same partition layout, same queries):
identical ids and bit-equal distances.  Cases follow
Tests/MetalANNSTests/IVFFlatSearchTests.swift (recall, nprobe >= nlist equals
brute force) plus ragged and empty lists."""
import numpy as np
import pytest

import bench
import meltan_b200 as mb
import oracle as O

pytestmark = pytest.mark.gpu

MET = [(mb.Metric.cosine, O.COSINE), (mb.Metric.l2, O.L2), (mb.Metric.innerProduct, O.IP)]


def build(ctx, v, cent, metric_o):
    assign = O.ivf_assign(v, cent, metric_o)
    off, ids, packed, pn = O.ivf_layout(v, assign, len(cent))
    part = mb.Partition(ctx, cent, packed, ids, off)
    return part, (off, ids, packed, pn)


def check(ctx, part, lay, cent, q, k, nprobe, mg, mo):
    off, ids, packed, pn = lay
    got = mb.IVFFlatSearch.search_arrays(ctx, q, part, k, nprobe, mg)
    want = O.ivf_search(cent, packed, pn, ids, off, q, k, nprobe, mo)
    np.testing.assert_array_equal(got[2], want[2])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0], want[0])


@pytest.mark.parametrize("mg,mo", MET)
def test_ivf_parity_small(ctx, mg, mo):
    v, q = bench.make_mixture(20000, 64, 50, 40, seed=1)
    rng = np.random.default_rng(2)
    cent = v[rng.choice(len(v), 64, replace=False)].copy()
    part, lay = build(ctx, v, cent, mo)
    for nprobe in (1, 4, 8, 63, 64, 1000):
        for k in (1, 10, 100):
            check(ctx, part, lay, cent, q[:1], k, nprobe, mg, mo)
            check(ctx, part, lay, cent, q, k, nprobe, mg, mo)
    part.close()


def test_ivf_empty_and_ragged_lists(ctx):
    v, q = bench.make_mixture(5000, 48, 8, 33, seed=3)
    rng = np.random.default_rng(4)
    cent = np.concatenate([v[rng.choice(len(v), 20, replace=False)],
                           rng.standard_normal((12, 48)).astype(np.float32) * 50])  # far: empty
    part, lay = build(ctx, v, cent, O.L2)
    assert (np.diff(lay[0]) == 0).any()
    for nprobe in (1, 3, 16, 31):
        check(ctx, part, lay, cent, q, 25, nprobe, mb.Metric.l2, O.L2)
    part.close()


def test_ivf_nprobe_all_equals_bruteforce(ctx):
    """IVFFlatSearchTests.swift:193-216."""
    v, q = bench.make_mixture(8000, 40, 16, 9, seed=5)
    cent = v[:32].copy()
    for mg, mo in MET:
        part, lay = build(ctx, v, cent, mo)
        got = mb.IVFFlatSearch.search_arrays(ctx, q, part, 30, 32, mg)
        want = O.flat_search(v, q, 30, mo)
        for a, b in zip(got, want):
            np.testing.assert_array_equal(a, b)
        part.close()


def test_ivf_recall_at_10(ctx):
    """IVFFlatSearchTests.swift:77-142 asks recall@10 >= 0.95 on clustered data
    (tight clusters, as the reference test's +-0.02 jitter around centres)."""
    v, q = bench.make_mixture(30000, 64, 64, 50, sigma=0.05, seed=6)
    cent, assign = bench.train_partition(v, 64, O.COSINE)
    part = mb.Partition.from_assignment(ctx, v, cent, assign)
    got = mb.IVFFlatSearch.search_arrays(ctx, q, part, 10, 8, mb.Metric.cosine)
    want = O.flat_search(v, q, 10, O.COSINE)
    rec = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(got[1], want[1])])
    assert rec >= 0.95
    part.close()


def test_ivf_single_query_api_and_errors(ctx):
    v, q = bench.make_mixture(3000, 32, 8, 2, seed=7)
    part, lay = build(ctx, v, v[:16].copy(), O.COSINE)
    res = mb.IVFFlatSearch.search(ctx, q[0], part, 5, 4, mb.Metric.cosine)
    assert len(res) == 5 and all(res[i].score <= res[i + 1].score for i in range(4))
    with pytest.raises(mb.DimensionMismatch):
        mb.IVFFlatSearch.search(ctx, q[0][:31], part, 5, 4, mb.Metric.cosine)
    with pytest.raises(mb.SearchFailed):
        mb.IVFFlatSearch.search_arrays(ctx, q, part, 5, 4, mb.Metric.hamming)
    assert mb.IVFFlatSearch.search(ctx, q[0], part, 0, 4, mb.Metric.cosine) == []
    part.close()


def _oracle_threads(fn, q, threads=16):
    """The oracle over query chunks on host threads (its ctypes calls
    release the GIL); results concatenated in query order."""
    from concurrent.futures import ThreadPoolExecutor
    parts = np.array_split(np.arange(len(q)), min(threads, len(q)))
    with ThreadPoolExecutor(len(parts)) as ex:
        outs = list(ex.map(lambda ix: fn(q[ix]), parts))
    return tuple(np.concatenate([o[j] for o in outs]) for j in range(3))


@pytest.mark.slow
def test_ivf_full_size_1m_x_384(ctx):
    """BASELINE config C3 at its own size: 1M x 384 mixture of 1024, nlist
    1024 (partition built on the device, as the bench builds it), nprobe
    4/8/32, cosine, k = 10 -- 8 single queries and one 256-query batch (the
    batch route: small-corpus centroid step and per-list query grouping),
    every query against the oracle's scanProbedLists."""
    v, q = bench.make_mixture(1_000_000, 384, 1024, 256 + 8, seed=0)
    cent = bench.train_centroids(v, 1024)
    buf = mb.VectorBuffer(ctx, v)
    part = mb.Partition.build(ctx, buf, cent, mb.Metric.cosine)
    off, order = part.layout()
    packed = v[order]
    pn = O.row_norms(packed)
    singles, batch = q[256:], q[:256]
    for nprobe in (4, 8, 32):
        want1 = O.ivf_search(cent, packed, pn, order, off, singles, 10, nprobe, O.COSINE)
        for i in range(len(singles)):
            got = mb.IVFFlatSearch.search_arrays(ctx, singles[i:i + 1], part, 10, nprobe,
                                                 mb.Metric.cosine)
            for a, b in zip(got, want1):
                np.testing.assert_array_equal(a[0], b[i])
        got = mb.IVFFlatSearch.search_arrays(ctx, batch, part, 10, nprobe, mb.Metric.cosine)
        want = _oracle_threads(lambda qq: O.ivf_search(cent, packed, pn, order, off, qq, 10,
                                                       nprobe, O.COSINE), batch)
        for a, b in zip(got, want):
            np.testing.assert_array_equal(a, b)
    part.close()
    buf.close()


@pytest.mark.parametrize("mg,mo", MET)
def test_gpu_partition_build_equals_host_layout(ctx, mg, mo):
    """buildPartition on the device (assignRows + counting-sort layout +
    packed rows): the assignment, offsets and list ids equal the oracle's
    restatement (IVFFlatSearch.swift:559-703), and searches match the oracle
    on that layout."""
    v, q = bench.make_mixture(30000, 48, 40, 21, seed=11)
    rng = np.random.default_rng(12)
    cent = v[rng.choice(len(v), 40, replace=False)] + np.float32(0.01)
    buf = mb.VectorBuffer(ctx, v)
    got_assign = mb.assign_rows(ctx, buf, cent, mg)
    want_assign = O.ivf_assign(v, cent, mo)
    np.testing.assert_array_equal(got_assign, want_assign)
    part = mb.Partition.build(ctx, buf, cent, mg)
    off, ids = part.layout()
    woff, wids, packed, pn = O.ivf_layout(v, want_assign, len(cent))
    np.testing.assert_array_equal(off, woff)
    np.testing.assert_array_equal(ids, wids)
    for nprobe in (1, 5, 40):
        got = mb.IVFFlatSearch.search_arrays(ctx, q, part, 10, nprobe, mg)
        want = O.ivf_search(cent, packed, pn, wids, woff, q, 10, nprobe, mo)
        for a, b in zip(got, want):
            np.testing.assert_array_equal(a, b)
    part.close()
    buf.close()


def test_gpu_partition_build_single_list_and_tiny(ctx):
    v, q = bench.make_mixture(700, 20, 3, 4, seed=13)
    buf = mb.VectorBuffer(ctx, v)
    for cent in (v[:1].copy(), v[:700:100].copy()):
        part = mb.Partition.build(ctx, buf, cent, mb.Metric.l2)
        off, ids = part.layout()
        woff, wids, _, _ = O.ivf_layout(v, O.ivf_assign(v, cent, O.L2), len(cent))
        np.testing.assert_array_equal(off, woff)
        np.testing.assert_array_equal(ids, wids)
        part.close()
    buf.close()
