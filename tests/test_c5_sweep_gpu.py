"""Exact-scan parity at the sizes of BASELINE config C5, the mixed-dimension
inner-product sweep: L2-normalised Gaussian rows, inner product, top-10, at
1M rows with d = 128, 768 and 1536 and at 10M rows with d = 128, each with
single queries and a 4096-query batch (the two ends of the HBM-bound to
tensor-bound crossover).

Single queries go through the path the library picks for them (the bf16
candidate pass with its exact fp32 re-rank, on corpora of 2^25 elements and
more) and are compared with the CPU oracle's exact top-k (the (distance, id)
order of FlatGPUSearch.swift:917-932, dots.c's sequential order): identical
ids, bit-equal distances.  The 4096-query batch runs the tensor-core path and is compared,
query by query, with the exact CUDA-core scan of the same batch, and a
sample of its queries with the oracle.

The rows are drawn on the device (torch's CUDA Philox generator, seeded), as
the bench draws inputs of 2^26 elements and more."""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import meltan_b200 as mb
import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

K = 10
NQ_BATCH = 4096


def _unit_rows(n, dim, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    out = np.empty((n, dim), np.float32)
    step = max(1, (1 << 26) // dim)
    for r0 in range(0, n, step):
        r1 = min(n, r0 + step)
        x = torch.randn((r1 - r0, dim), generator=g, device="cuda", dtype=torch.float32)
        x /= x.norm(dim=1, keepdim=True)
        out[r0:r1] = x.cpu().numpy()
    return out


def _oracle(v, q):
    """O.flat_search over the rows of q, one query per worker thread (the
    oracle's ctypes call releases the GIL)."""
    with ThreadPoolExecutor(len(q)) as ex:
        outs = list(ex.map(lambda i: O.flat_search(v, q[i:i + 1], K, O.IP), range(len(q))))
    return tuple(np.concatenate([o[j] for o in outs]) for j in range(3))


def _same(got, want):
    np.testing.assert_array_equal(got[2], want[2])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0], want[0])


def _check(ctx, n, dim, seed):
    v = _unit_rows(n, dim, seed)
    q = _unit_rows(NQ_BATCH, dim, seed + 1)
    buf = mb.VectorBuffer(ctx, v)
    try:
        singles = [2, 4095]
        got = [mb.FlatGPUSearch.batch_search_arrays(ctx, q[i:i + 1], buf, K, mb.Metric.innerProduct)
               for i in singles]
        got = tuple(np.concatenate([g[j] for g in got]) for j in range(3))
        pick = np.array([0, 1365, 2730])
        want = _oracle(v, q[np.concatenate([singles, pick])])
        _same(got, tuple(w[:len(singles)] for w in want))

        ctx.set_tensor_core_batch(16)
        tc = mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, K, mb.Metric.innerProduct)
        ctx.set_tensor_core_batch(0)
        exact = mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, K, mb.Metric.innerProduct)
        ctx.set_tensor_core_batch(16)
        _same(tc, exact)
        _same(tuple(a[pick] for a in tc), tuple(w[len(singles):] for w in want))
        # the single-query calls agree with the batch on the same queries
        _same(got, tuple(a[singles] for a in tc))
    finally:
        ctx.set_tensor_core_batch(16)
        buf.close()


@pytest.mark.parametrize("dim", [128, 768, 1536])
def test_c5_inner_product_1m_rows(ctx, dim):
    _check(ctx, 1_000_000, dim, seed=dim)


def test_c5_inner_product_10m_rows_d128(ctx):
    _check(ctx, 10_000_000, 128, seed=10)
