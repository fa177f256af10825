"""One context over several GPUs of one process (mans_ctx_create_multi): the
corpus is split into row shards, one per GPU, and mans_flat_search (host
buffers) searches them all, each GPU storing its shard's top-k into the first
GPU's memory, which merges them (ParallelFlatScan.mergeSorted over the
shards, ParallelFlatScan.swift:288-315).  Results must equal the oracle's
search of the whole corpus, ids and distances bit-equal.  Needs two GPUs
(skipped otherwise); the host-side split is the numpy.array_split rule checked
on CPU by test_shard_gloo.py."""
import time

import numpy as np
import pytest

import meltan_b200 as mb
import oracle as O
from tests.mann_files import write_mann

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.fixture(scope="module")
def group():
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    g = mb.Context.multi([0, 1])
    yield g
    g.close()


MET = [(mb.Metric.cosine, O.COSINE), (mb.Metric.l2, O.L2), (mb.Metric.innerProduct, O.IP)]


def same(got, want):
    for a, b in zip(got, want):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("mg,mo", MET)
def test_two_gpu_context_equals_oracle(group, mg, mo):
    """Shards of 15006 and 15005 rows; single queries (the exact scan on each
    shard) and a 40-query batch (the tensor-core pass on each shard)."""
    assert group.device_count == 2
    v = O.lcg_vectors(30011, 64, 51)
    q = O.lcg_vectors(40, 64, 52)
    buf = mb.VectorBuffer(group, v)
    assert buf.count == 30011
    for k in (1, 10, 100, 256):
        same(mb.FlatGPUSearch.batch_search_arrays(group, q[:1], buf, k, mg),
             O.flat_search(v, q[:1], k, mo))
        same(mb.FlatGPUSearch.batch_search_arrays(group, q, buf, k, mg),
             O.flat_search(v, q, k, mo))
    buf.close()


def test_two_gpu_context_device_order_and_small_corpus(group):
    """A corpus smaller than k per shard, and the devices listed in the other
    order (shard 0 on GPU 1, merged there)."""
    g10 = mb.Context.multi([1, 0])
    try:
        v = O.lcg_vectors(7, 16, 61)
        q = O.lcg_vectors(3, 16, 62)
        for ctx in (group, g10):
            buf = mb.VectorBuffer(ctx, v)
            same(mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, 10, mb.Metric.l2),
                 O.flat_search(v, q, 10, O.L2))
            buf.close()
    finally:
        g10.close()


def test_two_gpu_context_row_updates_across_the_shard_boundary(group):
    rng = np.random.default_rng(5)
    v = rng.standard_normal((4001, 32), dtype=np.float32)
    q = rng.standard_normal((5, 32), dtype=np.float32)
    buf = mb.VectorBuffer(group, v)
    new = rng.standard_normal((10, 32), dtype=np.float32) * np.float32(3)
    buf.batch_insert(new, 1995)  # rows 1995..2004 straddle the split at 2001
    v[1995:2005] = new
    same(mb.FlatGPUSearch.batch_search_arrays(group, q, buf, 20, mb.Metric.cosine),
         O.flat_search(v, q, 20, O.COSINE))
    codes, scales = buf.int8_codes()
    want_codes, want_scales = O.int8_fill(v)
    np.testing.assert_array_equal(codes, want_codes)
    np.testing.assert_array_equal(scales, want_scales)
    buf.close()


def test_two_gpu_context_loads_an_index_file(group, tmp_path):
    v = O.lcg_vectors(5003, 48, 3)
    q = O.lcg_vectors(4, 48, 4)
    path = tmp_path / "g.mann"
    write_mann(path, v, version=3)
    buf = mb.VectorBuffer.load_mann(group, path)
    same(mb.FlatGPUSearch.batch_search_arrays(group, q, buf, 10, mb.Metric.cosine),
         O.flat_search(v, q, 10, O.COSINE))
    buf.close()


def test_two_gpu_context_rejects_single_device_calls(group):
    with pytest.raises(mb.ConstructionFailed):
        mb.Workspace(group)
    v = O.lcg_vectors(100, 8, 1)
    with pytest.raises(mb.ConstructionFailed):
        mb.Partition.build(group, mb.VectorBuffer(group, v), v[:4].copy(), mb.Metric.l2)


def test_two_gpu_context_at_benchmark_size(group, ctx):
    """1M x 384 cosine, k = 10: the two-GPU context equals the single-GPU
    search (itself pinned to the oracle at this size) for single queries and
    a 1024-query batch; prints the end-to-end times of both."""
    rng = np.random.default_rng(0)
    v = rng.standard_normal((1_000_000, 384), dtype=np.float32)
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    q = rng.standard_normal((1024, 384), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    one = mb.VectorBuffer(ctx, v)
    two = mb.VectorBuffer(group, v)
    for nq in (1, 1024):
        want = mb.FlatGPUSearch.batch_search_arrays(ctx, q[:nq], one, 10, mb.Metric.cosine)
        same(mb.FlatGPUSearch.batch_search_arrays(group, q[:nq], two, 10, mb.Metric.cosine), want)
    for name, c, b in (("1 GPU", ctx, one), ("2 GPUs", group, two)):
        for nq, reps in ((1, 200), (1024, 20)):
            mb.FlatGPUSearch.batch_search_arrays(c, q[:nq], b, 10, mb.Metric.cosine)
            ts = []
            for r in range(reps):
                t = time.perf_counter()
                mb.FlatGPUSearch.batch_search_arrays(c, q[(r * nq) % 1024:][:nq] if nq == 1
                                                     else q, b, 10, mb.Metric.cosine)
                ts.append(time.perf_counter() - t)
            ts.sort()
            print(f"[multi-device] {name} nq={nq}: p50 {1e6 * ts[len(ts) // 2 - 1]:.1f} us, "
                  f"{nq * reps / sum(ts):.0f} queries/s end to end")
    one.close()
    two.close()
