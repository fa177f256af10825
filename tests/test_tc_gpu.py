"""GPU parity of the tensor-core batch path (bf16 tcgen05 candidate GEMM,
certified bound, exact fp32 re-score) against the CPU oracle: identical ids,
bit-equal distances.  A private context forces the path on for every batch
size; the exact CUDA-core scan is the cross-check at full size."""
import numpy as np
import pytest

import meltan_b200 as mb
import oracle as O

pytestmark = pytest.mark.gpu

MET = [(mb.Metric.cosine, O.COSINE), (mb.Metric.l2, O.L2), (mb.Metric.innerProduct, O.IP)]


@pytest.fixture(scope="module")
def tctx():
    c = mb.Context(0)
    c.set_tensor_core_batch(1)
    yield c
    c.close()


def unit_rows(rng, n, d):
    v = rng.standard_normal((n, d), dtype=np.float32)
    return v / np.linalg.norm(v, axis=1, keepdims=True)


def run(ctx, v, q, k, metric):
    buf = mb.VectorBuffer(ctx, v)
    try:
        return mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, k, metric)
    finally:
        buf.close()


def same(got, want):
    np.testing.assert_array_equal(got[2], want[2])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0], want[0])


@pytest.mark.parametrize("mg,mo", MET)
@pytest.mark.parametrize("n,d", [(1000, 32), (70001, 100), (20000, 384), (5000, 768),
                                 (3000, 1536)])
def test_tc_parity_small(tctx, mg, mo, n, d):
    rng = np.random.default_rng(n + d)
    v = unit_rows(rng, n, d)
    q = unit_rows(rng, 37, d)
    for k in (1, 10, 100):
        same(run(tctx, v, q, k, mg), O.flat_search(v, q, k, mo))


@pytest.mark.parametrize("n", [1, 7, 64, 255, 257])
def test_tc_tiny_corpora(tctx, n):
    """Corpora shorter than one 256-row tile (an IVF centroid table is one)."""
    rng = np.random.default_rng(n)
    v = unit_rows(rng, n, 64)
    q = unit_rows(rng, 20, 64)
    for mg, mo in MET:
        for k in (1, 10):
            same(run(tctx, v, q, k, mg), O.flat_search(v, q, k, mo))


def test_tc_many_query_blocks_wide_rows(tctx):
    """Five 128-query blocks over 1536-wide rows (queries streamed per tile)."""
    rng = np.random.default_rng(1536)
    v = unit_rows(rng, 4000, 1536)
    q = unit_rows(rng, 600, 1536)
    for mg, mo in (MET[0], MET[2]):
        same(run(tctx, v, q, 10, mg), O.flat_search(v, q, 10, mo))


def test_tc_unnormalised_rows_and_k256(tctx):
    rng = np.random.default_rng(7)
    v = rng.standard_normal((30000, 128), dtype=np.float32) * rng.uniform(0.5, 3, (30000, 1)).astype(np.float32)
    q = rng.standard_normal((300, 128), dtype=np.float32)  # two query blocks of 256
    for mg, mo in MET:
        same(run(tctx, v, q, 256, mg), O.flat_search(v, q, 256, mo))


def test_tc_lcg_reference_cases(tctx):
    """FlatSearchTests.batchParity data (n = 4200, 16 queries, k = 50)."""
    v = O.lcg_vectors(4200, 128, 31)
    q = O.lcg_vectors(16, 128, 77)
    same(run(tctx, v, q, 50, mb.Metric.cosine), O.flat_search(v, q, 50, O.COSINE))


def test_tc_duplicates_force_exact_fallback(tctx):
    """10,000 copies of one row nearest to every query overflow the candidate
    lists; the affected queries are re-scanned exactly and stay bit-equal."""
    import torch
    rng = np.random.default_rng(3)
    v = unit_rows(rng, 40000, 64)
    q = unit_rows(rng, 20, 64)
    v[5000:15000] = q[0]
    buf = mb.VectorBuffer(tctx, v)
    ws = mb.Workspace(tctx)
    dq = torch.from_numpy(q).cuda()
    od = torch.empty((20, 10), dtype=torch.float32, device="cuda")
    oi = torch.empty((20, 10), dtype=torch.int32, device="cuda")
    oc = torch.empty((20,), dtype=torch.int32, device="cuda")
    mb.FlatGPUSearch.search_device(tctx, buf, ws, dq.data_ptr(), 20, 10, mb.Metric.cosine,
                                   od.data_ptr(), oi.data_ptr(), oc.data_ptr())
    ws.check()
    assert ws.fallbacks() >= 1
    want = O.flat_search(v, q, 10, O.COSINE)
    same((od.cpu().numpy(), oi.cpu().numpy().view(np.uint32), oc.cpu().numpy()), want)
    ws.close()
    buf.close()


@pytest.fixture(scope="module")
def pair_ctx():
    """A context whose multi-block batches run the opt-in pair pass: the
    MANS_TC_PAIRS switch is read at the context's first multi-block batch,
    which runs here while it is set."""
    import os
    old = os.environ.get("MANS_TC_PAIRS")
    os.environ["MANS_TC_PAIRS"] = "1"
    c = mb.Context(0)
    c.set_tensor_core_batch(1)
    try:
        rng = np.random.default_rng(3)
        v = unit_rows(rng, 5000, 64)
        q = unit_rows(rng, 256, 64)
        same(run(c, v, q, 10, mb.Metric.cosine), O.flat_search(v, q, 10, O.COSINE))
    finally:
        if old is None:
            del os.environ["MANS_TC_PAIRS"]
        else:
            os.environ["MANS_TC_PAIRS"] = old
    yield c
    c.close()


@pytest.mark.parametrize("mg,mo", MET)
@pytest.mark.parametrize("nq,d", [(256, 384), (300, 128), (1000, 384)])
def test_tc_pair_pass(pair_ctx, mg, mo, nq, d):
    """Two or more query blocks with resident queries run the filtered pass
    as CTA pairs (M = 256 MMAs over two CTAs, each streaming half of every
    row tile); an odd number of query blocks leaves the last pair's second
    CTA without queries."""
    rng = np.random.default_rng(nq + d)
    v = unit_rows(rng, 30001, d)
    q = unit_rows(rng, nq, d)
    for k in (10, 100):
        same(run(pair_ctx, v, q, k, mg), O.flat_search(v, q, k, mo))


@pytest.mark.parametrize("mg,mo", MET[:2])
def test_tc_large_batch_wide_bands(tctx, mg, mo):
    """More queries than SMs (the one-wave re-rank with a 512-entry band
    buffer and the warp-per-query thresholds): 1,500 copies of one query's
    row make a band wider than the buffer (exact re-scan), 300 copies of
    another a band sorted in shared memory, duplicates of a third straddle
    the k-th rank (ties by id)."""
    import torch
    rng = np.random.default_rng(17)
    v = unit_rows(rng, 40000, 64)
    q = unit_rows(rng, 200, 64)
    v[2000:3500] = q[0]
    v[9000:9300] = q[1]
    v[30000:30007] = q[2]
    buf = mb.VectorBuffer(tctx, v)
    ws = mb.Workspace(tctx)
    dq = torch.from_numpy(q).cuda()
    od = torch.empty((200, 10), dtype=torch.float32, device="cuda")
    oi = torch.empty((200, 10), dtype=torch.int32, device="cuda")
    oc = torch.empty((200,), dtype=torch.int32, device="cuda")
    mb.FlatGPUSearch.search_device(tctx, buf, ws, dq.data_ptr(), 200, 10, mg,
                                   od.data_ptr(), oi.data_ptr(), oc.data_ptr())
    ws.check()
    assert ws.fallbacks() >= 1
    want = O.flat_search(v, q, 10, mo)
    same((od.cpu().numpy(), oi.cpu().numpy().view(np.uint32), oc.cpu().numpy()), want)
    ws.close()
    buf.close()


def test_tc_zero_rows_take_the_exact_scan(tctx):
    rng = np.random.default_rng(5)
    v = unit_rows(rng, 3000, 48)
    v[::50] = 0.0
    q = unit_rows(rng, 20, 48)
    for mg, mo in MET:
        same(run(tctx, v, q, 25, mg), O.flat_search(v, q, 25, mo))


def test_tc_row_update_invalidates_bf16_copy(tctx):
    rng = np.random.default_rng(11)
    v = unit_rows(rng, 8000, 64)
    q = unit_rows(rng, 24, 64)
    buf = mb.VectorBuffer(tctx, v)
    mb.FlatGPUSearch.batch_search_arrays(tctx, q, buf, 10, mb.Metric.cosine)
    rep = q[:3].copy()
    buf.batch_insert(rep, 100)
    v2 = v.copy()
    v2[100:103] = rep
    same(mb.FlatGPUSearch.batch_search_arrays(tctx, q, buf, 10, mb.Metric.cosine),
         O.flat_search(v2, q, 10, O.COSINE))
    buf.close()


@pytest.mark.slow
def test_tc_full_size_1m_x_384_batch_1024(ctx):
    """BASELINE config C2 at nq = 1024: the tensor-core path (default for
    batches) equals the exact CUDA-core scan for every query, and the oracle
    for a sample of queries, at k = 10 and 100."""
    rng = np.random.default_rng(0)
    v = unit_rows(rng, 1_000_000, 384)
    q = unit_rows(rng, 1024, 384)
    buf = mb.VectorBuffer(ctx, v)
    for k in (10, 100):
        ctx.set_tensor_core_batch(16)
        got = mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, k, mb.Metric.cosine)
        ctx.set_tensor_core_batch(0)
        ref = mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, k, mb.Metric.cosine)
        ctx.set_tensor_core_batch(16)
        same(got, ref)
        pick = np.arange(0, 1024, 128)
        same(tuple(a[pick] for a in got), O.flat_search(v, q[pick], k, O.COSINE))
    buf.close()


def test_tc_nonfinite_rows_match_the_exact_scan():
    """A NaN or infinite row voids the bf16 error bound: the batch goes to the
    exact CUDA-core scan, so both settings return the same lists."""
    rng = np.random.default_rng(9)
    v = unit_rows(rng, 6000, 64)
    v[17, 3] = np.nan
    v[4000, 0] = np.inf
    q = unit_rows(rng, 20, 64)
    c = mb.Context(0)
    try:
        for mg, _ in MET:
            c.set_tensor_core_batch(1)
            got = run(c, v, q, 10, mg)
            c.set_tensor_core_batch(0)
            ref = run(c, v, q, 10, mg)
            same(got, ref)
    finally:
        c.close()
