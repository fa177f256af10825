"""mans_flat_search_noalloc: the exact flat search for callers that may not
allocate device memory at search time (inside a stream capture, under a
framework that owns all GPU memory, or in a latency-critical loop).  Its
scratch is a fixed 4 MiB device array instead of a workspace.

The test drives the entry point through the C ABI on two calls in a row and
compares every output with the workspace-based mans_flat_search_device
(bit-equal, the tolerance used by all flat-scan tests).  It lives in its own
file, collected last, and runs alone or after the rest of the suite."""
import ctypes as C

import numpy as np
import pytest

import meltan_b200 as mb
from meltan_b200._lib import lib

pytestmark = pytest.mark.gpu


def _noalloc(ctx, buf, dq, nq, k, metric, od, oi, oc, stream=0):
    L = lib()
    fn = L.mans_flat_search_noalloc
    fn.restype = C.c_int32
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_int32,
                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    return fn(ctx.handle, buf.handle, C.c_void_p(dq), nq, k, int(metric), C.c_void_p(od),
              C.c_void_p(oi), C.c_void_p(oc), C.c_void_p(stream))


def _outputs(nq, k):
    import torch
    kout = min(k, mb.MAX_TOP_K)
    return (torch.full((nq, kout), -1.0, dtype=torch.float32, device="cuda"),
            torch.full((nq, kout), -1, dtype=torch.int32, device="cuda"),
            torch.full((nq,), -1, dtype=torch.int32, device="cuda"))


def test_no_alloc_matches_workspace_search_twice(ctx):
    import torch
    rng = np.random.default_rng(12)
    v = rng.standard_normal((60_000, 384), dtype=np.float32)
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    buf = mb.VectorBuffer(ctx, v)
    ws = mb.Workspace(ctx)
    cases = [(5, 100, mb.Metric.cosine), (1, 10, mb.Metric.cosine), (3, 17, mb.Metric.l2),
             (8, 256, mb.Metric.innerProduct)]
    for nq, k, metric in cases:
        q = rng.standard_normal((nq, 384), dtype=np.float32)
        dq = torch.from_numpy(q).cuda()
        want = _outputs(nq, k)
        mb.FlatGPUSearch.search_device(ctx, buf, ws, dq.data_ptr(), nq, k, metric,
                                       *(t.data_ptr() for t in want))
        ws.check()
        for _ in range(2):  # two calls in a row share (and reuse) the scratch array
            got = _outputs(nq, k)
            mb.check(_noalloc(ctx, buf, dq.data_ptr(), nq, k, metric,
                              *(t.data_ptr() for t in got)))
            torch.cuda.synchronize()
            for a, b in zip(got, want):
                assert torch.equal(a, b), (nq, k, metric)
    ws.close()
    buf.close()


def test_no_alloc_leaves_free_device_memory_unchanged(ctx):
    """After the first call on the device, a call takes no device memory:
    the free-memory figure is the same before and after it."""
    import torch
    rng = np.random.default_rng(5)
    v = rng.standard_normal((30_000, 128), dtype=np.float32)
    buf = mb.VectorBuffer(ctx, v)
    nq, k = 4, 10
    dq = torch.from_numpy(rng.standard_normal((nq, 128), dtype=np.float32)).cuda()
    out = _outputs(nq, k)
    mb.check(_noalloc(ctx, buf, dq.data_ptr(), nq, k, mb.Metric.l2, *(t.data_ptr() for t in out)))
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        mb.check(_noalloc(ctx, buf, dq.data_ptr(), nq, k, mb.Metric.l2,
                          *(t.data_ptr() for t in out)))
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert int(out[2].sum()) == nq * k
    buf.close()


def test_no_alloc_rejects_requests_beyond_its_scratch(ctx):
    import torch
    rng = np.random.default_rng(3)
    v = rng.standard_normal((4096, 64), dtype=np.float32)
    buf = mb.VectorBuffer(ctx, v)
    nq, k = 4000, 256  # 4000 x 256 candidate keys cannot fit in 4 MiB
    dq = torch.zeros((nq, 64), dtype=torch.float32, device="cuda")
    out = _outputs(nq, k)
    rc = _noalloc(ctx, buf, dq.data_ptr(), nq, k, mb.Metric.l2, *(t.data_ptr() for t in out))
    assert rc == 4  # MANS_ERR_OOM -> gpuResourceExhausted (degradeable)
    with pytest.raises(mb.GPUResourceExhausted, match="scratch"):
        mb.check(rc)
    buf.close()
