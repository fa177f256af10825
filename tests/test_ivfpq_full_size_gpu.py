"""IVF-PQ parity at the benchmarked configuration:
10M x 128 rows from a 4096-component Gaussian mixture, nlist 4096, m = 16
sub-quantisers x 256 centroids, nprobe 32, L2, k = 10.  The index is built
as the bench builds it (torch-trained coarse centroids and codebooks, codes
and lists from mans_pq_encode); every query of a 1024-query batch (the busy
batch route of the ADC kernel's warp-resident top-k) and of 32 single-query
calls is compared with the oracle's restatement of _IVFPQIndex.search
(Sources/MetalANNS/IVFPQIndex.swift:177-226): identical internal ids,
bit-equal scores, identical tie order."""
import types

import numpy as np
import pytest

import bench
import meltan_b200 as mb
import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _oracle_threads(fn, q, threads=16):
    from concurrent.futures import ThreadPoolExecutor
    parts = np.array_split(np.arange(len(q)), min(threads, len(q)))
    with ThreadPoolExecutor(len(parts)) as ex:
        outs = list(ex.map(lambda ix: fn(q[ix]), parts))
    return tuple(np.concatenate([o[j] for o in outs]) for j in range(3))


def test_ivfpq_c4_at_size(ctx):
    base = types.SimpleNamespace(workload="ivfpq", n=10_000_000, dim=128, metric="l2", k=10,
                                 nq=1024, nlist=4096, nprobe=32, components=4096, pq_m=16,
                                 pq_shard="list", transport="p2p")
    v, q, art = bench.build_index_data(base, 1024 + 32, mb=mb, ctx=ctx)
    del v
    ix = mb.IVFPQIndex(ctx, art["coarse"], art["codebooks"], art["codes"],
                       (art["offsets"], art["lists"]), metric=mb.Metric.l2)
    sizes = np.diff(art["offsets"])
    assert sizes.sum() == 10_000_000

    def want(qq):
        return O.ivfpq_search(art["coarse"], art["codebooks"], art["codes"], art["offsets"],
                              art["lists"], qq, 10, 32, O.L2)

    batch = q[:1024]
    got = ix.search_arrays(batch, 10, 32)
    ref = _oracle_threads(want, batch)
    for a, b in zip(got, ref):
        np.testing.assert_array_equal(a, b)
    assert (got[2] == 10).all()
    singles = q[1024:]
    ref1 = want(singles)
    for i in range(len(singles)):
        g = ix.search_arrays(singles[i:i + 1], 10, 32)
        for a, b in zip(g, ref1):
            np.testing.assert_array_equal(a[0], b[i])
    ix.close()
