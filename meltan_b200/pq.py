"""IVF-PQ search and single-list ADC over the C ABI.

* ``IVFPQIndex``   -- the search side of ``_IVFPQIndex`` (Sources/MetalANNS/
                      IVFPQIndex.swift:177-226) over a trained index: coarse
                      centroids, PQ codebooks, codes per internal id and the
                      inverted lists in insertion order.
* ``GPUADCSearch`` -- ``GPUADCSearch.computeDistances`` (Sources/MetalANNSCore/
                      GPUADCSearch.swift:35-173).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import lib
from .core import MAX_TOP_K, ConstructionFailed, Context, Metric, SearchResult, Workspace, check


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _vp(a):
    return C.c_void_p(a.ctypes.data)


class IVFPQIndex:
    def __init__(self, context: Context, coarse, codebooks, codes, inverted_lists,
                 metric: Metric = Metric.l2, list_positions=None):
        """coarse [nlist, dim]; codebooks [m, 256, dim/m]; codes [n, m] uint8 per
        internal id; inverted_lists: sequence of id arrays (insertion order) or
        (offsets, flat_ids)."""
        coarse = _f32(coarse)
        codebooks = _f32(codebooks)
        codes = np.ascontiguousarray(codes, np.uint8)
        if isinstance(inverted_lists, tuple):
            offsets, flat = inverted_lists
        else:
            sizes = [len(x) for x in inverted_lists]
            offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
            flat = np.concatenate([np.asarray(x, np.uint32) for x in inverted_lists]) \
                if len(inverted_lists) else np.zeros(0, np.uint32)
        offsets = np.ascontiguousarray(offsets, np.int64)
        flat = np.ascontiguousarray(flat, np.uint32)
        if codebooks.ndim != 3:
            raise ConstructionFailed("codebooks must be [m, ks, dim/m]")
        m, ks, sub = codebooks.shape
        pos = None if list_positions is None else np.ascontiguousarray(list_positions, np.uint32)
        h = C.c_void_p()
        check(lib().mans_ivfpq_create(context.handle, _vp(coarse), coarse.shape[0],
                                      coarse.shape[1], _vp(codebooks), m, ks, _vp(codes),
                                      codes.shape[0], _vp(offsets), _vp(flat),
                                      None if pos is None else _vp(pos), int(metric),
                                      C.byref(h)))
        self._h = h
        self.context = context
        self.dim = coarse.shape[1]
        self.nlist = coarse.shape[0]

    @property
    def handle(self):
        return self._h

    def search_arrays(self, queries, k: int, nprobe: int):
        q = _f32(np.atleast_2d(queries))
        nq, dim = q.shape
        kout = max(0, k)  # k wide: BoundedSortedList(capacity: k) has no cap beyond k
        od = np.empty((nq, kout), np.float32)
        oi = np.empty((nq, kout), np.uint32)
        oc = np.empty(nq, np.int32)
        check(lib().mans_ivfpq_search(self.context.handle, self._h, _vp(q), nq, dim, k, nprobe,
                                      _vp(od), _vp(oi), _vp(oc)))
        return od, oi, oc

    def search(self, query, k: int, nprobe: int):
        od, oi, oc = self.search_arrays([query], k, nprobe)
        return [SearchResult("", float(od[0, i]), int(oi[0, i])) for i in range(oc[0])]

    def search_device(self, ws: Workspace, d_queries: int, nq: int, k: int, nprobe: int,
                      d_out_dist: int, d_out_ids: int, d_out_counts: int, stream: int = 0):
        check(lib().mans_ivfpq_search_device(self.context.handle, self._h, ws.handle,
                                             C.c_void_p(d_queries), nq, k, nprobe,
                                             C.c_void_p(d_out_dist), C.c_void_p(d_out_ids),
                                             C.c_void_p(d_out_counts), C.c_void_p(stream)))

    def search_partial_device(self, ws: Workspace, d_queries: int, nq: int, k: int, nprobe: int,
                              d_block: int, stream: int = 0):
        """This shard's packed block [scores | seqs | ids | counts] (2k entries
        per query) for mans_ivfpq_resolve_device."""
        check(lib().mans_ivfpq_search_partial_device(
            self.context.handle, self._h, ws.handle, C.c_void_p(d_queries), nq, k, nprobe,
            C.c_void_p(d_block), C.c_void_p(stream)))

    @staticmethod
    def shard_lists(offsets, flat, r0: int, r1: int):
        """The inverted lists of the row shard [r0, r1) of a global index:
        (offsets, ids, positions in the global lists), insertion order kept."""
        offsets = np.asarray(offsets, np.int64)
        flat = np.asarray(flat, np.uint32)
        keep = (flat >= r0) & (flat < r1)
        lists = np.repeat(np.arange(len(offsets) - 1), np.diff(offsets))
        pos = np.arange(len(flat), dtype=np.int64) - offsets[lists]
        sizes = np.bincount(lists[keep], minlength=len(offsets) - 1)
        soff = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        return soff, flat[keep], pos[keep].astype(np.uint32)

    @staticmethod
    def shard_lists_by_list(offsets, flat, owned):
        """The whole inverted lists a list shard owns (`owned`: a boolean mask
        over the lists) of a global index: (offsets with every other list
        empty, ids, positions in the lists), insertion order kept.  A search
        of the shard builds distance tables only for probed lists it holds."""
        offsets = np.asarray(offsets, np.int64)
        flat = np.asarray(flat, np.uint32)
        owned = np.asarray(owned, bool)
        lists = np.repeat(np.arange(len(offsets) - 1), np.diff(offsets))
        keep = owned[lists]
        pos = np.arange(len(flat), dtype=np.int64) - offsets[lists]
        sizes = np.diff(offsets) * owned
        soff = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        return soff, flat[keep], pos[keep].astype(np.uint32)

    def close(self):
        if self._h:
            lib().mans_ivfpq_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def list_owners(sizes, world: int) -> np.ndarray:
    """Rank owning each inverted list when whole lists are spread over
    `world` shards: largest list first to the least-loaded rank (ties to the
    lower rank), the same answer on every rank."""
    sizes = np.asarray(sizes, np.int64)
    owner = np.empty(len(sizes), np.int32)
    load = np.zeros(world, np.int64)
    for lst in np.argsort(-sizes, kind="stable"):
        r = int(np.argmin(load))
        owner[lst] = r
        load[r] += sizes[lst]
    return owner


def partial_words(nq: int, k: int) -> int:
    """int32 words of one shard's IVF-PQ block."""
    kin = 2 * min(k, MAX_TOP_K)
    return nq * (3 * kin + 1)


def resolve_device(context: Context, ws: Workspace, d_blocks: int, n_blocks: int,
                   block_stride: int, nq: int, k: int, d_out_dist: int, d_out_ids: int,
                   d_out_counts: int, stream: int = 0):
    """Merge the shards' blocks and apply the BoundedSortedList outcome."""
    check(lib().mans_ivfpq_resolve_device(context.handle, ws.handle, C.c_void_p(d_blocks),
                                          n_blocks, block_stride, nq, k, C.c_void_p(d_out_dist),
                                          C.c_void_p(d_out_ids), C.c_void_p(d_out_counts),
                                          C.c_void_p(stream)))


def encode(context: Context, vectors, coarse, codebooks, metric: Metric = Metric.l2):
    """IVFPQIndex.add's encoding on the device: (codes [n, m] uint8, coarse
    assignment [n] int32) -- nearestCoarseCentroid (IVFPQIndex.swift:514-550)
    and ProductQuantizer.encode(vector:subtracting:) (ProductQuantizer.swift:
    120-169), bit-exact."""
    v = _f32(np.atleast_2d(vectors))
    coarse = _f32(coarse)
    cb = _f32(codebooks)
    m, ks, sub = cb.shape
    n, dim = v.shape
    codes = np.empty((n, m), np.uint8)
    assign = np.empty(n, np.int32)
    check(lib().mans_pq_encode(context.handle, _vp(v), n, dim, _vp(coarse), coarse.shape[0],
                               _vp(cb), m, ks, int(metric), _vp(codes), _vp(assign)))
    return codes, assign


class GPUADCSearch:
    @staticmethod
    def compute_distances(context: Context, query, codebooks, codes) -> np.ndarray:
        q = _f32(query)
        cb = _f32(codebooks)
        m, ks, sub = cb.shape
        codes = np.ascontiguousarray(codes, np.uint8).reshape(-1, m)
        out = np.empty(codes.shape[0], np.float32)
        check(lib().mans_pq_adc_list(context.handle, _vp(q), q.shape[0], _vp(cb), m, ks,
                                     _vp(codes), codes.shape[0], _vp(out)))
        return out
