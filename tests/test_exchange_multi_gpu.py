"""Peer-memory exchange (mans_exchange) on two GPUs: row shards searched on
their own GPUs, blocks gathered over NVLink and merged in one kernel, equal to
the oracle's search of the whole corpus; many calls in a row exercise both
parities of the slots.  Needs two GPUs (skipped otherwise); the host logic of
the split and the packed block is covered on CPU by test_shard_gloo.py."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    import meltan_b200 as mb
    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        n, dim, nq, k = 30011, 64, 6, 10
        v = O.lcg_vectors(n, dim, 91)
        q = O.lcg_vectors(nq, dim, 92)
        ctx = mb.Context(rank)
        r0, r1 = mb.row_shard(n, world, rank)
        buf = mb.VectorBuffer(ctx, v[r0:r1], id_offset=r0)
        ws = mb.Workspace(ctx)
        sh = mb.ShardedFlatSearch(ctx, buf, world, dist, transport="p2p", rank=rank)
        bufs = sh.buffers(nq, k)
        dq = torch.from_numpy(q).cuda()
        results = []
        for it in range(7):
            out = sh.search_device(ws, dq.data_ptr(), nq, k, mb.Metric.cosine, bufs)
            ws.check()
            results.append(out.cpu().numpy().copy())
        torch.cuda.synchronize()
        dist.barrier()
        sh.close()
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.stack(results))
        ws.close()
        buf.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_two_gpu_peer_exchange_equals_unsharded(tmp_path):
    import torch
    import torch.multiprocessing as mp

    import oracle as O
    from meltan_b200 import shard

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    n, dim, nq, k = 30011, 64, 6, 10
    want = O.flat_search(O.lcg_vectors(n, dim, 91), O.lcg_vectors(nq, dim, 92), k, O.COSINE)
    for rank in range(2):
        res = np.load(tmp_path / f"r{rank}.npy")
        for blk in res:
            d, i, c = shard.block_views(torch.from_numpy(blk), nq, k)
            np.testing.assert_array_equal(c.numpy(), want[2])
            np.testing.assert_array_equal(i.numpy().view(np.uint32), want[1])
            np.testing.assert_array_equal(d.numpy(), want[0])


def _ivf_worker(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    import bench
    import meltan_b200 as mb

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        v, q = bench.make_mixture(40000, 48, 30, 9, seed=21)
        cent = v[::1000][:30].copy()
        ctx = mb.Context(rank)
        r0, r1 = mb.row_shard(len(v), world, rank)
        buf = mb.VectorBuffer(ctx, v[r0:r1], id_offset=r0)
        part = mb.Partition.build(ctx, buf, cent, mb.Metric.cosine)
        ws = mb.Workspace(ctx)
        sh = mb.ShardedIVFSearch(ctx, part, world, dist, transport="p2p", rank=rank)
        bufs = sh.buffers(len(q), 10)
        dq = torch.from_numpy(q).cuda()
        res = []
        for nprobe in (1, 4, 30):
            out = sh.search_device(ws, dq.data_ptr(), len(q), 10, nprobe, mb.Metric.cosine, bufs)
            ws.check()
            res.append(out.cpu().numpy().copy())
        torch.cuda.synchronize()
        dist.barrier()
        sh.close()
        np.save(os.path.join(out_dir, f"ivf{rank}.npy"), np.stack(res))
        part.close()
        ws.close()
        buf.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_ivf_equals_unsharded(tmp_path):
    """IVF-flat over row shards (each rank's partition of its rows under the
    same centroids, global ids) merged over peer memory equals the oracle's
    scanProbedLists on the whole corpus."""
    import torch
    import torch.multiprocessing as mp

    import bench
    import oracle as O
    from meltan_b200 import shard

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_ivf_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    v, q = bench.make_mixture(40000, 48, 30, 9, seed=21)
    cent = v[::1000][:30].copy()
    off, ids, packed, pn = O.ivf_layout(v, O.ivf_assign(v, cent, O.COSINE), len(cent))
    for rank in range(2):
        res = np.load(tmp_path / f"ivf{rank}.npy")
        for blk, nprobe in zip(res, (1, 4, 30)):
            want = O.ivf_search(cent, packed, pn, ids, off, q, 10, nprobe, O.COSINE)
            d, i, c = shard.block_views(torch.from_numpy(blk), len(q), 10)
            np.testing.assert_array_equal(c.numpy(), want[2])
            np.testing.assert_array_equal(i.numpy().view(np.uint32), want[1])
            np.testing.assert_array_equal(d.numpy(), want[0])


def _skip_worker(rank, world, port, out_dir):
    """Rank 1 skips the third exchange: rank 0's merge waits on a flag that
    nothing sets, gives up after its bounded wait (2 s) and must report the
    failure -- empty results and MANS_ERR_EXEC from the workspace check --
    instead of merging its own block alone."""
    import datetime

    import torch
    import torch.distributed as dist

    import meltan_b200 as mb
    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        n, dim, nq, k = 20000, 32, 3, 10
        v = O.lcg_vectors(n, dim, 71)
        q = O.lcg_vectors(nq, dim, 72)
        ctx = mb.Context(rank)
        r0, r1 = mb.row_shard(n, world, rank)
        buf = mb.VectorBuffer(ctx, v[r0:r1], id_offset=r0)
        ws = mb.Workspace(ctx)
        sh = mb.ShardedFlatSearch(ctx, buf, world, dist, transport="p2p", rank=rank)
        bufs = sh.buffers(nq, k)
        dq = torch.from_numpy(q).cuda()
        status = []
        counts = []
        for it in range(3):
            if not (rank == 1 and it == 2):  # rank 1 never publishes its third block
                out = sh.search_device(ws, dq.data_ptr(), nq, k, mb.Metric.l2, bufs)
                try:
                    ws.check()
                    status.append(0)
                except mb.GPUExecutionFailed:
                    status.append(5)
                counts.append(out[2 * nq * k:].cpu().numpy().copy())
            dist.barrier()  # the next exchange starts only when both ranks are done
        torch.cuda.synchronize()
        dist.barrier()
        sh.close()
        np.save(os.path.join(out_dir, f"skip{rank}.npy"),
                np.array([status + [-1] * (3 - len(status)),
                          [int(c.sum()) for c in counts] + [-1] * (3 - len(counts))]))
        ws.close()
        buf.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_peer_that_never_publishes_gives_empty_results_and_exec_error(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.start_processes(_skip_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    st0, counts0 = np.load(tmp_path / "skip0.npy")
    st1, counts1 = np.load(tmp_path / "skip1.npy")
    assert st0.tolist() == [0, 0, 5]          # the third merge timed out on rank 0
    assert counts0.tolist()[:2] == [30, 30]   # 3 queries x k = 10 while both publish
    assert counts0.tolist()[2] == 0           # ... and nothing once the peer is missing
    assert st1.tolist() == [0, 0, -1]
