"""GPU parity of the one-launch IVF-flat search (a few queries, k <= 32)
against the oracle's restatement of IVFFlatSearch.scanProbedLists: identical
ids, bit-equal distances, equal counts.  Every case also checks that the
search ran as one library launch, so the cooperative kernel (not the
six-launch batch path) produced the result, and that the host-buffer entry
point returns the same."""
import numpy as np
import pytest
import torch

import bench
import meltan_b200 as mb
import oracle as O

pytestmark = pytest.mark.gpu

MET = [(mb.Metric.cosine, O.COSINE), (mb.Metric.l2, O.L2), (mb.Metric.innerProduct, O.IP)]


def layout(v, cent, mo):
    assign = O.ivf_assign(v, cent, mo)
    return O.ivf_layout(v, assign, len(cent))


def run_device(ctx, part, q, k, nprobe, mg):
    """mans_ivf_search_device on torch buffers; returns the results and the
    number of library launches of the call."""
    q = np.ascontiguousarray(q, np.float32)
    nq = len(q)
    kout = min(k, 256)
    dq = torch.from_numpy(q).cuda()
    dd = torch.empty((nq, kout), dtype=torch.float32, device="cuda")
    di = torch.empty((nq, kout), dtype=torch.int32, device="cuda")
    dc = torch.empty(nq, dtype=torch.int32, device="cuda")
    ws = mb.Workspace(ctx)
    ws.set_timing(True)
    torch.cuda.synchronize()
    mb.IVFFlatSearch.search_device(ctx, part, ws, dq.data_ptr(), nq, k, nprobe, mg,
                                   dd.data_ptr(), di.data_ptr(), dc.data_ptr(), 0)
    ws.check(0)
    _, _, launches = ws.stats()
    ws.close()
    return (dd.cpu().numpy(), di.cpu().numpy().view(np.uint32), dc.cpu().numpy()), launches


def check(ctx, part, lay, cent, q, k, nprobe, mg, mo, fused=True):
    off, ids, packed, pn = lay
    got, launches = run_device(ctx, part, q, k, nprobe, mg)
    want = O.ivf_search(cent, packed, pn, ids, off, q, k, nprobe, mo)
    np.testing.assert_array_equal(got[2], want[2])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0], want[0])
    if fused:
        assert launches == 1, f"expected the one-launch path, saw {launches} launches"
    host = mb.IVFFlatSearch.search_arrays(ctx, q, part, k, nprobe, mg)
    for a, b in zip(host, want):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("mg,mo", MET)
def test_probe_metrics_batches_and_k(ctx, mg, mo):
    v, q = bench.make_mixture(40000, 96, 128, 4, seed=21)
    rng = np.random.default_rng(22)
    cent = v[rng.choice(len(v), 128, replace=False)].copy()
    lay = layout(v, cent, mo)
    part = mb.Partition(ctx, cent, lay[2], lay[1], lay[0])
    for nq in (1, 2, 3, 4):
        for k in (1, 10, 32):
            for nprobe in (1, 4, 8, 127):
                check(ctx, part, lay, cent, q[:nq], k, nprobe, mg, mo)
    part.close()


@pytest.mark.parametrize("dim", [3, 33, 130, 384, 768])
def test_probe_dims(ctx, dim):
    v, q = bench.make_mixture(6000, dim, 40, 3, seed=dim)
    cent = v[:: len(v) // 40][:40].copy()
    lay = layout(v, cent, O.COSINE)
    part = mb.Partition(ctx, cent, lay[2], lay[1], lay[0])
    for nprobe in (1, 7, 39):
        check(ctx, part, lay, cent, q, 10, nprobe, mb.Metric.cosine, O.COSINE)
        check(ctx, part, lay, cent, q[:1], 10, nprobe, mb.Metric.cosine, O.COSINE)
    part.close()


def test_probe_many_lists(ctx):
    """nlist above 32 x SMs: every block scores two centroid tiles."""
    rng = np.random.default_rng(23)
    v = rng.standard_normal((60000, 16), dtype=np.float32)
    q = rng.standard_normal((4, 16), dtype=np.float32)
    cent = rng.standard_normal((8192, 16), dtype=np.float32)
    lay = layout(v, cent, O.L2)
    part = mb.Partition(ctx, cent, lay[2], lay[1], lay[0])
    for nprobe in (1, 16, 256):
        check(ctx, part, lay, cent, q[:1], 10, nprobe, mb.Metric.l2, O.L2)
        check(ctx, part, lay, cent, q, 32, nprobe, mb.Metric.l2, O.L2)
    part.close()


def test_probe_tiny_empty_and_ragged(ctx):
    """Fewer rows than blocks, empty lists (far centroids) and k above the
    candidate count."""
    rng = np.random.default_rng(24)
    v = rng.standard_normal((50, 24), dtype=np.float32)
    q = rng.standard_normal((3, 24), dtype=np.float32)
    cent = np.concatenate([v[:6], rng.standard_normal((6, 24)).astype(np.float32) * 100])
    lay = layout(v, cent, O.L2)
    assert (np.diff(lay[0]) == 0).any()
    part = mb.Partition(ctx, cent, lay[2], lay[1], lay[0])
    for nprobe in (1, 2, 6, 11):
        for k in (1, 5, 32):
            check(ctx, part, lay, cent, q, k, nprobe, mb.Metric.l2, O.L2)
    part.close()


def test_probe_ties(ctx):
    """Duplicate rows (equal distances order by id) and duplicate centroids
    (equal centroid keys: the lower list index is probed)."""
    rng = np.random.default_rng(25)
    base = rng.standard_normal((300, 32), dtype=np.float32)
    v = np.concatenate([base] * 20)  # every row 20 times
    q = np.concatenate([base[:2], rng.standard_normal((2, 32), dtype=np.float32)])
    cent = base[:24].copy()
    cent[5] = cent[3]
    cent[17] = cent[3]
    for mg, mo in MET:
        lay = layout(v, cent, mo)
        part = mb.Partition(ctx, cent, lay[2], lay[1], lay[0])
        for nprobe in (1, 2, 3, 4):
            check(ctx, part, lay, cent, q, 32, nprobe, mg, mo)
        part.close()


def test_probe_boundaries_take_other_paths(ctx):
    """k above 32, five queries and nprobe >= nlist take the other paths;
    results still equal the oracle."""
    v, q = bench.make_mixture(8000, 48, 32, 5, seed=26)
    cent = v[:32].copy()
    lay = layout(v, cent, O.COSINE)
    part = mb.Partition(ctx, cent, lay[2], lay[1], lay[0])
    check(ctx, part, lay, cent, q[:1], 33, 4, mb.Metric.cosine, O.COSINE, fused=False)
    check(ctx, part, lay, cent, q, 10, 4, mb.Metric.cosine, O.COSINE, fused=False)
    check(ctx, part, lay, cent, q[:1], 10, 32, mb.Metric.cosine, O.COSINE, fused=False)
    part.close()


def test_probe_repeated_calls_share_counters(ctx):
    """The grid-barrier and arrival counters carry over between calls on one
    workspace: many calls in a row keep giving the oracle's answer."""
    v, q = bench.make_mixture(20000, 64, 64, 8, seed=27)
    cent = v[:64].copy()
    off, ids, packed, pn = layout(v, cent, O.COSINE)
    part = mb.Partition(ctx, cent, packed, ids, off)
    want = O.ivf_search(cent, packed, pn, ids, off, q, 10, 8, O.COSINE)
    ws = mb.Workspace(ctx)
    dq = torch.from_numpy(q).cuda()
    dd = torch.empty((1, 10), dtype=torch.float32, device="cuda")
    di = torch.empty((1, 10), dtype=torch.int32, device="cuda")
    dc = torch.empty(1, dtype=torch.int32, device="cuda")
    for rep in range(40):
        i = rep % len(q)
        mb.IVFFlatSearch.search_device(ctx, part, ws, dq[i].data_ptr(), 1, 10, 8,
                                       mb.Metric.cosine, dd.data_ptr(), di.data_ptr(),
                                       dc.data_ptr(), 0)
        ws.check(0)
        np.testing.assert_array_equal(di.cpu().numpy().view(np.uint32)[0], want[1][i])
        np.testing.assert_array_equal(dd.cpu().numpy()[0], want[0][i])
    ws.close()
    part.close()


@pytest.mark.parametrize("mg,mo", MET)
def test_batch_segment_scan(ctx, mg, mo):
    """Query batches (5 or more queries, k <= 32) take the warp-per-segment
    list scan: segments of up to four queries of one list.  Many queries on
    one list (the same query repeated), k at the edge of the path (32, and
    33 on the streaming scan) and several dims."""
    for dim in (3, 130, 384):
        v, q = bench.make_mixture(12000, dim, 48, 40, seed=30 + dim)
        cent = v[:: len(v) // 48][:48].copy()
        lay = layout(v, cent, mo)
        part = mb.Partition(ctx, cent, lay[2], lay[1], lay[0])
        qq = np.concatenate([q, np.repeat(q[:1], 23, axis=0)])  # one list, 24 queries
        for k in (1, 10, 32, 33):
            for nprobe in (1, 5, 47):
                check(ctx, part, lay, cent, qq, k, nprobe, mg, mo, fused=False)
        part.close()
