"""Host-side mirror of the MetalANNS search-path interface over the C ABI.

Names, argument meaning and error behaviour follow the reference Swift types
(paths relative to the MetalANNS source tree):

* ``Metric``             -- Sources/MetalANNSCore/Metric.swift:1-6, codes of
                            FlatGPUSearch.swift:134-140
* ``ANNSError``          -- Sources/MetalANNSCore/Errors.swift:6-31
* ``SearchResult``       -- Sources/MetalANNSCore/SearchResult.swift:1-13
* ``Context``            -- MetalContext (MetalDevice.swift:9-111)
* ``VectorBuffer``       -- VectorBuffer.swift:12-111 (row-major fp32 corpus)
* ``FlatGPUSearch``      -- FlatGPUSearch.swift:12-181 (search / batchSearch /
                            isEligible)

All computation runs in ``libmans_cuda.so``; this module only validates,
marshals and maps status codes to exceptions.
"""
from __future__ import annotations

import ctypes as C
import os
import enum
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

from ._lib import last_error, lib

MAX_TOP_K = 256
EMPTY_ID = 0xFFFFFFFF
TC_AUTO, TC_BF16, TC_INT8 = 0, 1, 2  # MANS_TC_* operand formats


class Metric(enum.IntEnum):
    cosine = 0
    l2 = 1
    innerProduct = 2
    hamming = 3


# ---- errors (Errors.swift:6-31) ---------------------------------------------


class ANNSError(Exception):
    degradeable = False

    @property
    def is_tier_degradeable(self) -> bool:
        """Errors.swift:23-30: pipeline, resource, execution and search failures."""
        return self.degradeable


class DimensionMismatch(ANNSError):
    pass


class SearchFailed(ANNSError):
    degradeable = True


class GPUPipelineUnavailable(ANNSError):
    degradeable = True


class GPUResourceExhausted(ANNSError):
    degradeable = True


class GPUExecutionFailed(ANNSError):
    degradeable = True


class ConstructionFailed(ANNSError):
    pass


class DeviceNotSupported(ANNSError):
    pass


class CorruptFile(ANNSError):
    """ANNSError.corruptFile (Errors.swift:11): a malformed index file."""


_STATUS = {
    1: DimensionMismatch,
    2: SearchFailed,
    3: GPUPipelineUnavailable,
    4: GPUResourceExhausted,
    5: GPUExecutionFailed,
    6: ConstructionFailed,
    7: DeviceNotSupported,
    8: CorruptFile,
}


def check(status: int) -> None:
    if status != 0:
        raise _STATUS.get(status, ANNSError)(last_error())


@dataclass
class SearchResult:
    id: str
    score: float
    internalID: int


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray):
    return C.c_void_p(a.ctypes.data)


# ---- context / storage ----------------------------------------------------------


class Context:
    """One CUDA device; stands in for MetalContext.  ``Context.multi(devices)``
    makes one context over several GPUs of this process: a VectorBuffer
    created on it holds one row shard per GPU and FlatGPUSearch searches them
    all, merging on the first GPU (mans_ctx_create_multi)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().mans_ctx_create(device, C.byref(h)))
        self._h = h
        self.device = device

    @classmethod
    def multi(cls, devices):
        devs = (C.c_int32 * len(devices))(*devices)
        h = C.c_void_p()
        check(lib().mans_ctx_create_multi(devs, len(devices), C.byref(h)))
        self = cls.__new__(cls)
        self._h = h
        self.device = devices[0]
        return self

    @property
    def device_count(self) -> int:
        return lib().mans_ctx_device_count(self._h)

    @property
    def handle(self):
        return self._h

    @property
    def sm_count(self) -> int:
        return lib().mans_ctx_sm_count(self._h)

    def set_tensor_core_batch(self, min_batch: int) -> None:
        """Batches of >= min_batch queries use the tensor-core path (0: never)."""
        check(lib().mans_ctx_set_tensor_core_batch(self._h, min_batch))

    def set_tensor_core_format(self, fmt: int) -> None:
        """Operand format of the tensor-core path: TC_AUTO, TC_BF16 or TC_INT8."""
        check(lib().mans_ctx_set_tensor_core_format(self._h, fmt))

    def close(self):
        if self._h:
            lib().mans_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MannInfo(C.Structure):
    """mans_mann_info: header and section offsets of a reference index file."""
    _fields_ = [(name, C.c_uint32) for name in
                ("version", "count", "degree", "dim", "metric", "storage", "page_size",
                 "idmap_bytes", "entry_point")] + \
               [(name, C.c_uint64) for name in
                ("vector_offset", "vector_bytes", "adjacency_offset", "distance_offset",
                 "idmap_offset")]


def mann_info(path) -> MannInfo:
    """Parses a reference index file (IndexSerializer versions 1-3)."""
    info = MannInfo()
    check(lib().mans_mann_read_info(os.fsencode(path), C.byref(info)))
    return info


class VectorBuffer:
    """Device-resident row-major fp32 corpus with cached squared norms."""

    def __init__(self, context: Context, vectors, id_offset: int = 0):
        v = _f32(vectors)
        if v.ndim != 2:
            raise ConstructionFailed("vectors must be a 2-D array")
        self.context = context
        h = C.c_void_p()
        check(lib().mans_corpus_create(context.handle, _ptr(v), v.shape[0], v.shape[1],
                                       id_offset, C.byref(h)))
        self._h = h
        self.id_offset = id_offset

    @classmethod
    def load_mann(cls, context: Context, path, shard_index: int = 0, shard_count: int = 1):
        """Vector section of a reference index file (loadReadOnly(.mmap)):
        rows of shard `shard_index` of `shard_count`, ids offset by the shard's
        first row."""
        self = cls.__new__(cls)
        h = C.c_void_p()
        check(lib().mans_corpus_load_mann(context.handle, os.fsencode(path), shard_index,
                                          shard_count, C.byref(h)))
        self._h = h
        self.context = context
        info = mann_info(path)
        base, extra = divmod(info.count, shard_count)
        self.id_offset = shard_index * base + min(shard_index, extra)
        return self

    @property
    def handle(self):
        return self._h

    @property
    def count(self) -> int:
        return lib().mans_corpus_count(self._h)

    @property
    def dim(self) -> int:
        return lib().mans_corpus_dim(self._h)

    def insert(self, vector, at: int) -> None:
        """In-place row write; norms refresh on the device (VectorBuffer.swift:57-91)."""
        self.batch_insert(np.atleast_2d(vector), at)

    def batch_insert(self, vectors, starting_at: int) -> None:
        v = _f32(np.atleast_2d(vectors))
        if v.shape[1] != self.dim:
            raise DimensionMismatch(f"expected {self.dim}, got {v.shape[1]}")
        check(lib().mans_corpus_update_rows(self._h, starting_at, _ptr(v), v.shape[0]))

    def int8_codes(self):
        """(codes [n, dim] int8, scales [n]) of the int8 prefilter copy, as
        Int8CodeBuffer.fill quantises the rows (Int8CodeCache.swift:64-99)."""
        n, d = self.count, self.dim
        codes = np.empty((n, d), np.int8)
        scales = np.empty(n, np.float32)
        check(lib().mans_corpus_int8_codes(self._h, C.c_void_p(codes.ctypes.data),
                                           C.c_void_p(scales.ctypes.data)))
        return codes, scales

    def close(self):
        if self._h:
            lib().mans_corpus_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Workspace:
    """Scratch for device-pointer calls (one in-flight call at a time)."""

    def __init__(self, context: Context):
        h = C.c_void_p()
        check(lib().mans_workspace_create(context.handle, C.byref(h)))
        self._h = h
        self.context = context

    @property
    def handle(self):
        return self._h

    def check(self, stream_ptr: int = 0) -> None:
        check(lib().mans_workspace_check(self._h, C.c_void_p(stream_ptr)))

    def fallbacks(self) -> int:
        out = C.c_int32()
        check(lib().mans_workspace_fallbacks(self._h, C.byref(out)))
        return out.value

    def last_path(self) -> int:
        """Path of the last flat search: 0 scan, 1 bf16 tensor core, 2 int8."""
        out = C.c_int32()
        check(lib().mans_workspace_last_path(self._h, C.byref(out)))
        return out.value

    def set_timing(self, enable: bool, stages: bool = False) -> None:
        """Dominant-kernel timing (`enable`) and per-stage timing (`stages`)
        of the searches made with this workspace."""
        check(lib().mans_workspace_set_timing(self._h, (1 if enable else 0) | (2 if stages else 0)))

    STAGES = ("query_prep", "sample", "threshold", "pass", "rerank", "merge")

    def stage_times(self):
        """{stage: (summed ms, timed launches)} since per-stage timing was
        enabled or last read (waits for the timed work)."""
        n = len(self.STAGES)
        ms = (C.c_double * n)()
        cnt = (C.c_int64 * n)()
        check(lib().mans_workspace_stage_times(self._h, ms, cnt, n))
        return {name: (ms[i], cnt[i]) for i, name in enumerate(self.STAGES)}

    def stats(self):
        """(summed dominant-kernel ms, timed launches, all library launches)."""
        ms = C.c_double()
        kl = C.c_int64()
        tl = C.c_int64()
        check(lib().mans_workspace_stats(self._h, C.byref(ms), C.byref(kl), C.byref(tl)))
        return ms.value, kl.value, tl.value

    def close(self):
        if self._h:
            lib().mans_workspace_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- FlatGPUSearch --------------------------------------------------------------


class FlatGPUSearch:
    """Exact flat search (FlatGPUSearch.swift).  Results ascend by (distance, id)."""

    maxTopK = MAX_TOP_K
    minEligibleVectorCount = 64  # FlatGPUSearch.swift:15

    @staticmethod
    def is_eligible(vectors: VectorBuffer, metric: Metric, k: int, max_vector_count: int) -> bool:
        """FlatGPUSearch.isEligible (FlatGPUSearch.swift:193-205)."""
        if metric == Metric.hamming:
            return False
        if not (1 <= k <= MAX_TOP_K):
            return False
        if vectors.count < FlatGPUSearch.minEligibleVectorCount:
            return False
        return max_vector_count > 0 and vectors.count <= max_vector_count

    @staticmethod
    def batch_search_arrays(context: Context, queries, vectors: VectorBuffer, k: int,
                            metric: Metric):
        """Array form of batchSearch: (dist[nq, kout], ids[nq, kout], counts[nq])."""
        q = _f32(np.atleast_2d(queries))
        nq, dim = q.shape
        kout = max(0, min(k, MAX_TOP_K))
        od = np.empty((nq, kout), np.float32)
        oi = np.empty((nq, kout), np.uint32)
        oc = np.empty(nq, np.int32)
        check(lib().mans_flat_search(context.handle, vectors.handle, _ptr(q), nq, dim, k,
                                     int(metric), _ptr(od), _ptr(oi), _ptr(oc)))
        return od, oi, oc

    @staticmethod
    def batch_search(context: Context, queries: Sequence, vectors: VectorBuffer, k: int,
                     metric: Metric) -> List[List[SearchResult]]:
        """FlatGPUSearch.batchSearch (FlatGPUSearch.swift:103-181)."""
        if len(queries) == 0:
            return []
        if k <= 0:
            return [[] for _ in queries]
        if vectors.count == 0:
            return [[] for _ in queries]
        if metric == Metric.hamming:
            raise SearchFailed("FlatGPUSearch does not support metric .hamming")
        for q in queries:
            if len(q) != vectors.dim:
                raise DimensionMismatch(f"expected {vectors.dim}, got {len(q)}")
        od, oi, oc = FlatGPUSearch.batch_search_arrays(context, np.asarray(queries), vectors, k,
                                                       metric)
        return [[SearchResult("", float(od[r, i]), int(oi[r, i])) for i in range(oc[r])]
                for r in range(len(queries))]

    @staticmethod
    def search(context: Optional[Context], query, vectors: VectorBuffer, k: int,
               metric: Metric) -> List[SearchResult]:
        """FlatGPUSearch.search for one query (GPU tier)."""
        if context is None:
            raise DeviceNotSupported("no CUDA context")
        out = FlatGPUSearch.batch_search(context, [list(query)], vectors, k, metric)
        if not out:
            raise SearchFailed("FlatGPUSearch produced no results")
        return out[0]

    @staticmethod
    def search_device(context: Context, vectors: VectorBuffer, ws: Workspace, d_queries: int,
                      nq: int, k: int, metric: Metric, d_out_dist: int, d_out_ids: int,
                      d_out_counts: int, stream: int = 0) -> None:
        """Device-pointer search enqueued on `stream` (no synchronisation)."""
        check(lib().mans_flat_search_device(context.handle, vectors.handle, ws.handle,
                                            C.c_void_p(d_queries), nq, k, int(metric),
                                            C.c_void_p(d_out_dist), C.c_void_p(d_out_ids),
                                            C.c_void_p(d_out_counts), C.c_void_p(stream)))


def topk_merge_device(context: Context, ws: Workspace, d_in_dist: int, d_in_ids: int,
                      d_in_counts: int, n_lists: int, nq: int, kin: int, k: int,
                      d_out_dist: int, d_out_ids: int, d_out_counts: int, stream: int = 0,
                      list_stride: int = 0):
    """Merge of row-shard result blocks by (distance, id) (mergeSorted semantics).
    list_stride (4-byte elements) locates block l of all three inputs at
    base + l * list_stride; 0 means plain list-major arrays."""
    check(lib().mans_topk_merge_device(context.handle, ws.handle, C.c_void_p(d_in_dist),
                                       C.c_void_p(d_in_ids), C.c_void_p(d_in_counts), n_lists,
                                       list_stride, nq, kin, k, C.c_void_p(d_out_dist),
                                       C.c_void_p(d_out_ids), C.c_void_p(d_out_counts),
                                       C.c_void_p(stream)))
