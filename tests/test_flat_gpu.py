"""GPU parity of the exact flat scan against the CPU oracle.

Distances are compared bit-for-bit (the kernels use the reference's sequential
fp32 dot order and host-tier formulas) and ids exactly, with ties ordered by
id.  Cases follow Tests/MetalANNSTests/FlatSearchTests.swift,
ExactSearchIntegrationTests.swift and BoundedSelectionTests.swift.
"""
import numpy as np
import pytest

import meltan_b200 as mb
import oracle as O

pytestmark = pytest.mark.gpu

MET = {"cosine": (mb.Metric.cosine, O.COSINE), "l2": (mb.Metric.l2, O.L2),
       "ip": (mb.Metric.innerProduct, O.IP)}


def gpu_search(ctx, corpus, queries, k, metric):
    buf = mb.VectorBuffer(ctx, corpus)
    try:
        return mb.FlatGPUSearch.batch_search_arrays(ctx, queries, buf, k, metric)
    finally:
        buf.close()


def assert_same(got, want):
    gd, gi, gc = got
    wd, wi, wc = want
    np.testing.assert_array_equal(gc, wc)
    np.testing.assert_array_equal(gi, wi)
    # bit-exact distances (-0.0 and +0.0 compare equal)
    np.testing.assert_array_equal(gd, wd)


@pytest.mark.parametrize("n", [64, 100, 2048, 2049, 5000])
@pytest.mark.parametrize("metric", ["cosine", "l2", "ip"])
def test_flat_parity_across_metrics_and_sizes(ctx, n, metric):
    """FlatSearchTests.parityAcrossMetricsAndSizes (FlatSearchTests.swift:73-115)."""
    v = O.lcg_vectors(n, 128, n)
    q = O.lcg_vectors(1, 128, n + 999)
    mg, mo = MET[metric]
    assert_same(gpu_search(ctx, v, q, 100, mg), O.flat_search(v, q, 100, mo))


def test_flat_batch_parity(ctx):
    """FlatSearchTests.batchParity (FlatSearchTests.swift:117-148)."""
    v = O.lcg_vectors(4200, 128, 31)
    q = O.lcg_vectors(16, 128, 77)
    assert_same(gpu_search(ctx, v, q, 50, mb.Metric.cosine), O.flat_search(v, q, 50, O.COSINE))


def test_k_exceeds_corpus(ctx):
    """FlatSearchTests.kExceedsCorpus (FlatSearchTests.swift:150-169)."""
    v = O.lcg_vectors(70, 32, 7)
    q = O.lcg_vectors(1, 32, 5)
    got = gpu_search(ctx, v, q, 256, mb.Metric.l2)
    assert got[2][0] == 70
    assert_same(got, O.flat_search(v, q, 256, O.L2))


@pytest.mark.parametrize("dim", [1, 3, 4, 5, 31, 32, 33, 100, 383, 384, 385, 768, 1536])
def test_dimensions_including_ragged_tails(ctx, dim):
    v = O.lcg32_vectors(777, dim, dim)
    q = O.lcg32_vectors(3, dim, dim + 1)
    for mg, mo in MET.values():
        assert_same(gpu_search(ctx, v, q, 17, mg), O.flat_search(v, q, 17, mo))


@pytest.mark.parametrize("n", [1, 2, 31, 32, 33, 255, 256, 257, 511, 513, 70001])
def test_row_counts_around_tile_edges(ctx, n):
    v = O.lcg_vectors(n, 64, 1000 + n)
    q = O.lcg_vectors(2, 64, 7)
    for k in (1, 10, 256):
        assert_same(gpu_search(ctx, v, q, k, mb.Metric.cosine), O.flat_search(v, q, k, O.COSINE))


@pytest.mark.parametrize("nq", [1, 2, 3, 4, 5, 8, 9, 17, 33])
def test_query_batch_widths(ctx, nq):
    v = O.lcg_vectors(9000, 96, 42)
    q = O.lcg_vectors(nq, 96, 43)
    for k in (1, 10, 100):
        assert_same(gpu_search(ctx, v, q, k, mb.Metric.l2), O.flat_search(v, q, k, O.L2))


def test_norm_cache_refresh_after_in_place_write(ctx):
    """FlatSearchTests.normCacheInvalidation (FlatSearchTests.swift:171-206)."""
    v = O.lcg_vectors(512, 64, 13)
    q = O.lcg_vectors(1, 64, 21)
    buf = mb.VectorBuffer(ctx, v)
    mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, 20, mb.Metric.cosine)
    mutated = v.copy()
    for row in (3, 100, 411):
        rep = O.lcg_vectors(1, 64, row + 500)[0]
        buf.insert(rep, row)
        mutated[row] = rep
    for mg, mo in (MET["cosine"], MET["l2"]):
        assert_same(mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, 25, mg),
                    O.flat_search(mutated, q, 25, mo))
    buf.close()


def test_duplicate_vectors_tie_order_by_id(ctx):
    """BoundedSelectionTests.gpuTierTieOrderPinned (:257-277): ties ascend by id."""
    base = O.lcg_vectors(6, 8, 11)
    v = np.repeat(base, 2, axis=0)
    q = O.lcg_vectors(1, 8, 99)
    for mg, mo in MET.values():
        got = gpu_search(ctx, v, q, 12, mg)
        assert_same(got, O.flat_search(v, q, 12, mo))
        ids = got[1][0].tolist()
        for a in range(0, 12, 2):
            assert ids[a] + 1 == ids[a + 1]


def test_many_exact_ties_and_zero_rows(ctx):
    # zero rows: cosine denominator below 1e-10 -> distance 1; IP gives -0
    v = np.zeros((300, 16), np.float32)
    v[::7] = O.lcg_vectors(43, 16, 3)
    q = O.lcg_vectors(2, 16, 4)
    for mg, mo in MET.values():
        assert_same(gpu_search(ctx, v, q, 256, mg), O.flat_search(v, q, 256, mo))


def test_empty_and_invalid_requests(ctx):
    v = O.lcg_vectors(100, 16, 1)
    buf = mb.VectorBuffer(ctx, v)
    d, i, c = mb.FlatGPUSearch.batch_search_arrays(ctx, O.lcg_vectors(2, 16, 2), buf, 0,
                                                   mb.Metric.l2)
    assert d.shape == (2, 0) and list(c) == [0, 0]
    with pytest.raises(mb.SearchFailed):
        mb.FlatGPUSearch.batch_search_arrays(ctx, O.lcg_vectors(1, 16, 2), buf, 5,
                                             mb.Metric.hamming)
    with pytest.raises(mb.DimensionMismatch):
        mb.FlatGPUSearch.batch_search_arrays(ctx, O.lcg_vectors(1, 15, 2), buf, 5, mb.Metric.l2)
    assert mb.FlatGPUSearch.batch_search(ctx, [], buf, 5, mb.Metric.l2) == []
    res = mb.FlatGPUSearch.search(ctx, O.lcg_vectors(1, 16, 9)[0], buf, 3, mb.Metric.cosine)
    assert len(res) == 3 and res[0].score <= res[1].score <= res[2].score
    buf.close()
    empty = mb.VectorBuffer(ctx, np.zeros((0, 16), np.float32))
    d, i, c = mb.FlatGPUSearch.batch_search_arrays(ctx, O.lcg_vectors(1, 16, 2), empty, 5,
                                                   mb.Metric.l2)
    assert c[0] == 0 and np.all(i == mb.EMPTY_ID) and np.all(np.isinf(d))
    empty.close()


def test_device_api_and_shard_merge(ctx):
    """Row shards searched separately and merged on the device equal the
    unsharded search (the all-gather + mergeSorted path)."""
    import torch
    n, dim, nq, k = 20000, 64, 5, 10
    v = O.lcg_vectors(n, dim, 77)
    q = O.lcg_vectors(nq, dim, 78)
    cuts = [0, 7001, 13000, n]
    shards = [mb.VectorBuffer(ctx, v[a:b], id_offset=a) for a, b in zip(cuts, cuts[1:])]
    ws = mb.Workspace(ctx)
    dq = torch.from_numpy(q).cuda()
    L = len(shards)
    dd = torch.empty((L, nq, k), dtype=torch.float32, device="cuda")
    di = torch.empty((L, nq, k), dtype=torch.int32, device="cuda")
    dc = torch.empty((L, nq), dtype=torch.int32, device="cuda")
    for s, buf in enumerate(shards):
        mb.FlatGPUSearch.search_device(ctx, buf, ws, dq.data_ptr(), nq, k, mb.Metric.cosine,
                                       dd[s].data_ptr(), di[s].data_ptr(), dc[s].data_ptr())
    od = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    oi = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    oc = torch.empty((nq,), dtype=torch.int32, device="cuda")
    mb.topk_merge_device(ctx, ws, dd.data_ptr(), di.data_ptr(), dc.data_ptr(), L, nq, k, k,
                         od.data_ptr(), oi.data_ptr(), oc.data_ptr())
    ws.check()
    want = O.flat_search(v, q, k, O.COSINE)
    got = (od.cpu().numpy(), oi.cpu().numpy().view(np.uint32), oc.cpu().numpy())
    assert_same(got, want)
    # packed per-shard blocks [dist | ids | counts], merged with a list stride
    P = 2 * nq * k + nq
    packed = torch.empty((L, P), dtype=torch.int32, device="cuda")
    for s_, buf in enumerate(shards):
        base = packed[s_]
        mb.FlatGPUSearch.search_device(ctx, buf, ws, dq.data_ptr(), nq, k, mb.Metric.cosine,
                                       base.data_ptr(), base[nq * k:].data_ptr(),
                                       base[2 * nq * k:].data_ptr())
    mb.topk_merge_device(ctx, ws, packed.data_ptr(), packed[0, nq * k:].data_ptr(),
                         packed[0, 2 * nq * k:].data_ptr(), L, nq, k, k, od.data_ptr(),
                         oi.data_ptr(), oc.data_ptr(), list_stride=P)
    ws.check()
    got = (od.cpu().numpy(), oi.cpu().numpy().view(np.uint32), oc.cpu().numpy())
    assert_same(got, want)
    ws.close()
    for b in shards:
        b.close()


@pytest.mark.slow
def test_full_size_1m_x_384_cosine(ctx):
    """The benchmark configuration (1M x 384, L2-normalised Gaussian, cosine),
    bit-exact against the oracle for a few queries at k = 10 and 100."""
    rng = np.random.default_rng(0)
    v = rng.standard_normal((1_000_000, 384), dtype=np.float32)
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    q = rng.standard_normal((3, 384), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    buf = mb.VectorBuffer(ctx, v)
    for k in (10, 100):
        got = mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, k, mb.Metric.cosine)
        assert_same(got, O.flat_search(v, q, k, O.COSINE))
    buf.close()
