"""The oracle's restatement of KMeans.cluster's Lloyd loop
(Sources/MetalANNSCore/KMeans.swift:95-254) against an independent
pure-Python statement of the same steps (fp32 scalars, the reference's
per-chunk sums added in chunk order, strict '<' assignment, stop before the
update when nothing changed, sum * (1 / count)), on cases small enough for
Python loops: both the sequential path (workers 1, n < 512 or k < 8) and the
chunked path of useParallelLloyd (:89-190)."""
import numpy as np
import pytest

import oracle as O

F32_MAX = np.float32(np.finfo(np.float32).max)


def lloyd_py(v, cent, iters, metric, workers, offset=0, dim=None):
    n = v.shape[0]
    dim = v.shape[1] - offset if dim is None else dim
    x = np.ascontiguousarray(v[:, offset:offset + dim], np.float32)
    cent = np.array(cent, np.float32, copy=True)
    k = cent.shape[0]
    w = min(max(1, workers), n)
    if not (w > 1 and n >= 512 and k >= 8):
        w = 1
    chunk = -(-n // w)
    assign = [-1] * n
    updates = 0
    for _ in range(iters):
        sums = [[[np.float32(0)] * dim for _ in range(k)] for _ in range(w)]
        counts = [[0] * k for _ in range(w)]
        changed = False
        for i in range(n):
            best, bd = 0, F32_MAX
            for c in range(k):
                d = np.float32(O.simd_distance(x[i], cent[c], metric))
                if d < bd:
                    bd, best = d, c
            if assign[i] != best:
                changed = True
            assign[i] = best
            wi = i // chunk
            counts[wi][best] += 1
            acc = sums[wi][best]
            for d in range(dim):
                acc[d] = np.float32(acc[d] + x[i, d])
        if not changed:
            break
        for c in range(k):
            cnt = sum(counts[wi][c] for wi in range(w))
            if cnt == 0:
                continue
            scale = np.float32(np.float32(1.0) / np.float32(cnt))
            for d in range(dim):
                total = np.float32(0)
                for wi in range(w):
                    total = np.float32(total + sums[wi][c][d])
                cent[c, d] = np.float32(total * scale)
        updates += 1
    return cent, np.asarray(assign, np.int32), updates


@pytest.mark.parametrize("n,dim,k,workers,metric,iters", [
    (120, 6, 5, 4, O.L2, 6),        # n < 512: one running sum
    (600, 5, 8, 4, O.L2, 5),        # chunked sums (4 chunks of 150)
    (600, 5, 9, 7, O.COSINE, 4),    # uneven chunks (86 rows, last one shorter)
    (520, 4, 8, 16, O.IP, 3),
    (530, 3, 6, 8, O.L2, 4),        # k < 8: sequential even with workers
])
def test_oracle_lloyd_equals_python_statement(n, dim, k, workers, metric, iters):
    rng = np.random.default_rng(n + dim + k)
    v = rng.standard_normal((n, dim), dtype=np.float32)
    init = v[rng.choice(n, k, replace=False)] + np.float32(0.01)
    got = O.kmeans_lloyd(v, init, iters, metric, workers)
    want = lloyd_py(v, init, iters, metric, workers)
    np.testing.assert_array_equal(got[0], want[0])
    np.testing.assert_array_equal(got[1], want[1])
    assert got[2] == want[2]


def test_oracle_lloyd_subspace_empty_cluster_and_convergence():
    rng = np.random.default_rng(3)
    v = rng.standard_normal((560, 12), dtype=np.float32)
    init = np.concatenate([v[:7, 4:8], np.full((1, 4), 100, np.float32)])  # cluster 7 stays empty
    got = O.kmeans_lloyd(v, init, 30, O.L2, 4, offset=4, dim=4)
    want = lloyd_py(v, init, 30, O.L2, 4, offset=4, dim=4)
    np.testing.assert_array_equal(got[0], want[0])
    np.testing.assert_array_equal(got[1], want[1])
    assert got[2] == want[2] and got[2] < 30   # converged: stopped before the limit
    np.testing.assert_array_equal(got[0][7], init[7])  # an empty cluster keeps its centroid
    assert not (got[1] == 7).any()
