"""Row sharding of the exact flat search, one process per GPU.

The corpus rows are split contiguously: rank r holds rows [r0, r1) and
reports global ids (r0 + local row, through the corpus ``id_offset``).  Each
rank's per-query top-k is written into one int32 block

    [ distances (nq * kout float32 bits) | ids (nq * kout uint32) | counts (nq) ]

so that a single all-gather moves every rank's lists; the gathered blocks are
then merged by (distance, id) on the device (``topk_merge_device`` with
``list_stride`` = the block size).  This is the slice-and-merge structure of
``ParallelFlatScan.search`` (Sources/MetalANNSCore/ParallelFlatScan.swift:
96-155 slices, 288-315 ``mergeSorted``) with GPUs in place of host threads.
"""
from __future__ import annotations

import ctypes as C

from . import core
from ._lib import lib

__all__ = ["row_shard", "packed_words", "block_views", "all_gather_blocks", "PeerExchange",
           "ShardedFlatSearch", "ShardedIVFSearch", "ShardedIVFPQSearch"]


def row_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of ``rank``: the first n % world ranks hold one extra row
    (the split of ``numpy.array_split``)."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def packed_words(nq: int, kout: int) -> int:
    """int32 words of one rank's packed block."""
    return 2 * nq * kout + nq


def block_views(block, nq: int, kout: int):
    """(distances, ids, counts) views of one packed block (a 1-D int32 torch
    tensor); the distance view reinterprets the words as float32."""
    import torch

    if block.dim() != 1 or block.dtype != torch.int32 or block.numel() != packed_words(nq, kout):
        raise ValueError("block must be a 1-D int32 tensor of packed_words(nq, kout) words")
    d = block[: nq * kout].view(torch.float32).view(nq, kout)
    i = block[nq * kout: 2 * nq * kout].view(nq, kout)
    c = block[2 * nq * kout:]
    return d, i, c


def all_gather_blocks(dist, local_block, gathered):
    """One collective: ``gathered[r]`` = rank r's block (a (world, words)
    tensor).  Every rank calls it in the same order."""
    if gathered.dim() != 2 or gathered.shape[1] != local_block.numel():
        raise ValueError("gathered must be (world, words)")
    if gathered.shape[0] == 1:
        gathered[0].copy_(local_block)
        return gathered
    # the concatenated 1-D form is accepted by both NCCL and gloo
    dist.all_gather_into_tensor(gathered.view(-1), local_block)
    return gathered


class PeerExchange:
    """mans_exchange: the packed blocks of all ranks gathered over NVLink peer
    memory and merged in one kernel (CUDA IPC handles shared once through
    ``dist.all_gather_object``).  Every rank calls ``allgather`` in the same
    order."""

    HANDLE_BYTES = 64

    def __init__(self, ctx, world: int, rank: int, max_block_words: int, dist):
        h = C.c_void_p()
        core.check(lib().mans_exchange_create(ctx.handle, world, rank, max_block_words,
                                              C.byref(h)))
        self._h = h
        mine = (C.c_uint8 * self.HANDLE_BYTES)()
        core.check(lib().mans_exchange_handle(h, mine))
        handles = [None] * world
        dist.all_gather_object(handles, bytes(mine))
        flat = (C.c_uint8 * (self.HANDLE_BYTES * world)).from_buffer_copy(b"".join(handles))
        core.check(lib().mans_exchange_open(h, flat))

    def allgather(self, ws, block_ptr: int, nq: int, kin: int, k: int, out_dist: int,
                  out_ids: int, out_counts: int, stream: int = 0):
        core.check(lib().mans_exchange_allgather(
            self._h, ws.handle, C.c_void_p(block_ptr), nq, kin, k, C.c_void_p(out_dist),
            C.c_void_p(out_ids), C.c_void_p(out_counts), C.c_void_p(stream)))

    def close(self):
        if self._h:
            lib().mans_exchange_destroy(self._h)
            self._h = None


class _ShardedSearch:
    """Per-rank packed block -> every rank's block -> merged top-k."""

    def __init__(self, ctx, world: int, dist=None, transport: str = "nccl", rank: int = 0):
        self.ctx, self.world, self.dist = ctx, world, dist
        self.transport = transport if world > 1 else "none"
        self.rank = rank
        self._ex = {}

    def _exchange(self, words: int):
        ex = self._ex.get(words)
        if ex is None:
            ex = self._ex[words] = PeerExchange(self.ctx, self.world, self.rank, words, self.dist)
        return ex

    def buffers(self, nq: int, kout: int):
        """(local block, gathered blocks, merged block) device tensors."""
        import torch

        P = packed_words(nq, kout)
        loc = torch.empty((P,), dtype=torch.int32, device="cuda")
        gat = torch.empty((self.world, P), dtype=torch.int32, device="cuda")
        out = torch.empty((P,), dtype=torch.int32, device="cuda")
        return loc, gat, out

    def _local_target(self, bufs):
        loc, _, out = bufs
        return loc if self.world > 1 else out

    def _gather_merge(self, ws, bufs, nq: int, kout: int, k: int, stream: int):
        loc, gat, out = bufs
        if self.world == 1:
            return out
        if self.transport == "p2p":
            self._exchange(packed_words(nq, kout)).allgather(
                ws, loc.data_ptr(), nq, kout, k, out.data_ptr(), out[nq * kout:].data_ptr(),
                out[2 * nq * kout:].data_ptr(), stream)
            return out
        all_gather_blocks(self.dist, loc, gat)
        core.topk_merge_device(self.ctx, ws, gat.data_ptr(), gat[0, nq * kout:].data_ptr(),
                               gat[0, 2 * nq * kout:].data_ptr(), self.world, nq, kout, k,
                               out.data_ptr(), out[nq * kout:].data_ptr(),
                               out[2 * nq * kout:].data_ptr(), stream,
                               list_stride=packed_words(nq, kout))
        return out

    def close(self):
        for ex in self._ex.values():
            ex.close()
        self._ex = {}


class ShardedFlatSearch(_ShardedSearch):
    """Exact flat search over a row-sharded corpus: this rank's shard is a
    ``VectorBuffer`` created with ``id_offset`` = its first global row.  The
    per-rank blocks move by peer-memory exchange (``transport="p2p"``) or by
    one NCCL all-gather (``"nccl"``)."""

    def __init__(self, ctx, shard: "core.VectorBuffer", world: int, dist=None,
                 transport: str = "nccl", rank: int = 0):
        super().__init__(ctx, world, dist, transport, rank)
        self.shard = shard

    def search_device(self, ws, d_queries: int, nq: int, k: int, metric, bufs,
                      stream: int = 0):
        """Search this rank's shard, gather every rank's block and merge;
        returns the merged packed block (identical on every rank)."""
        kout = min(k, core.MAX_TOP_K)
        t = self._local_target(bufs)
        core.FlatGPUSearch.search_device(self.ctx, self.shard, ws, d_queries, nq, k, metric,
                                         t.data_ptr(), t[nq * kout:].data_ptr(),
                                         t[2 * nq * kout:].data_ptr(), stream)
        return self._gather_merge(ws, bufs, nq, kout, k, stream)


class ShardedIVFSearch(_ShardedSearch):
    """IVF-flat over row shards: every rank holds the partition of its rows
    under the same centroids (``Partition.build`` on a shard ``VectorBuffer``
    reports global ids), so every rank probes the same lists; the per-rank
    top-k blocks merge by (distance, id) into the unsharded result."""

    def __init__(self, ctx, partition, world: int, dist=None, transport: str = "nccl",
                 rank: int = 0):
        super().__init__(ctx, world, dist, transport, rank)
        self.partition = partition

    def search_device(self, ws, d_queries: int, nq: int, k: int, nprobe: int, metric, bufs,
                      stream: int = 0):
        from .ivf import IVFFlatSearch

        kout = min(k, core.MAX_TOP_K)
        t = self._local_target(bufs)
        IVFFlatSearch.search_device(self.ctx, self.partition, ws, d_queries, nq, k, nprobe,
                                    metric, t.data_ptr(), t[nq * kout:].data_ptr(),
                                    t[2 * nq * kout:].data_ptr(), stream)
        return self._gather_merge(ws, bufs, nq, kout, k, stream)


class ShardedIVFPQSearch:
    """IVF-PQ over row shards: every rank holds the same coarse centroids and
    codebooks and its rows' list entries with their global list positions;
    each search writes the shard's (score, sequence, id) block, one
    all-gather moves the blocks, and ``mans_ivfpq_resolve_device`` merges
    them and applies the BoundedSortedList outcome -- the unsharded result."""

    def __init__(self, ctx, index_shard, world: int, dist=None):
        self.ctx, self.index, self.world, self.dist = ctx, index_shard, world, dist

    def buffers(self, nq: int, k: int):
        import torch

        from .pq import partial_words

        w = partial_words(nq, k)
        loc = torch.empty((w,), dtype=torch.int32, device="cuda")
        gat = torch.empty((self.world, w), dtype=torch.int32, device="cuda")
        out = torch.empty((packed_words(nq, min(k, core.MAX_TOP_K)),), dtype=torch.int32,
                          device="cuda")
        return loc, gat, out

    def search_device(self, ws, d_queries: int, nq: int, k: int, nprobe: int, bufs,
                      stream: int = 0):
        from .pq import resolve_device

        loc, gat, out = bufs
        kout = min(k, core.MAX_TOP_K)
        self.index.search_partial_device(ws, d_queries, nq, k, nprobe, loc.data_ptr(), stream)
        all_gather_blocks(self.dist, loc, gat)
        resolve_device(self.ctx, ws, gat.data_ptr(), self.world, gat.shape[1], nq, k,
                       out.data_ptr(), out[nq * kout:].data_ptr(), out[2 * nq * kout:].data_ptr(),
                       stream)
        return out

    def close(self):
        pass
