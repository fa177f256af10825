"""ctypes front end of the CPU oracle (test infrastructure only).

The functions here wrap ``oracle/libmans_oracle.so`` (the C restatement of the
MetalANNS search path, see ``mans_oracle.c``) and, when it was built,
``oracle/_ref/libmans_ref_dots.so`` (the reference's own ``dots.c``).  Only the
test suite, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs use
this package; the CUDA product path never imports it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

COSINE, L2, IP, HAMMING = 0, 1, 2, 3
MAX_TOPK = 256

_F = C.POINTER(C.c_float)
_U32 = C.POINTER(C.c_uint32)
_I32 = C.POINTER(C.c_int32)
_I64 = C.POINTER(C.c_int64)
_U8 = C.POINTER(C.c_uint8)
DOT_ROWS_FN = C.CFUNCTYPE(None, _F, _F, C.c_int64, C.c_int64, _F)

_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        path = _build.ORACLE_SO
        if not os.path.exists(path):
            _build.build_oracle()
        L = C.CDLL(path)
        L.orc_lcg_vectors.argtypes = [C.c_uint64, C.c_int64, C.c_int64, _F]
        L.orc_lcg32_vectors.argtypes = [C.c_uint64, C.c_int64, C.c_int64, _F]
        L.orc_int8_fill.argtypes = [_F, C.c_int64, C.c_int64, C.c_void_p, _F]
        for name in ("orc_dot_rows_seq", "orc_dot_rows_neon"):
            getattr(L, name).argtypes = [_F, _F, C.c_int64, C.c_int64, _F]
        L.orc_norm_sq.argtypes = [_F, C.c_int64]
        L.orc_norm_sq.restype = C.c_float
        L.orc_row_norms.argtypes = [_F, C.c_int64, C.c_int64, _F]
        L.orc_distance.argtypes = [C.c_int32, C.c_float, C.c_float, C.c_float]
        L.orc_distance.restype = C.c_float
        L.orc_flat_search.argtypes = [_F, _F, C.c_int64, C.c_int64, _F, C.c_int64, C.c_int32,
                                      C.c_int32, C.c_void_p, _F, _U32, _I32]
        L.orc_parallel_flat_scan.argtypes = [_F, _F, _F, C.c_float, C.c_int64, C.c_int64,
                                             C.c_int32, C.c_int32, C.c_int32, C.c_void_p, _F, _U32]
        L.orc_parallel_flat_scan.restype = C.c_int
        L.orc_gpu_tier_topk.argtypes = [_F, C.c_int64, C.c_int32, _F, _U32]
        L.orc_gpu_tier_topk.restype = C.c_int
        L.orc_ivf_assign.argtypes = [_F, _F, C.c_int64, C.c_int64, _F, _F, C.c_int32, C.c_int32, _I32]
        L.orc_ivf_layout.argtypes = [_F, _F, C.c_int64, C.c_int64, _I32, C.c_int32, _I64, _U32, _F, _F]
        L.orc_ivf_search.argtypes = [_F, _F, C.c_int32, _F, _F, _U32, _I64, C.c_int64, C.c_int64,
                                     _F, C.c_int64, C.c_int32, C.c_int32, C.c_int32, _F, _U32, _I32]
        L.orc_simd_distance.argtypes = [_F, _F, C.c_int64, C.c_int32]
        L.orc_simd_distance.restype = C.c_float
        L.orc_pq_lut.argtypes = [_F, _F, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _F]
        L.orc_pq_encode_subtracting.argtypes = [_F, _F, _F, C.c_int32, C.c_int32, C.c_int32, _U8]
        L.orc_nearest_coarse.argtypes = [_F, _F, C.c_int32, C.c_int64, C.c_int32]
        L.orc_nearest_coarse.restype = C.c_int32
        L.orc_ivfpq_search.argtypes = [_F, C.c_int32, C.c_int64, _F, C.c_int32, C.c_int32, _U8,
                                       _I64, _U32, _F, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                                       _F, _U32, _I32]
        L.orc_pq_adc.argtypes = [_F, C.c_int32, C.c_int32, _U8, C.c_int64, _F]
        L.orc_kmeans_lloyd.argtypes = [_F, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int32,
                                       C.c_int32, C.c_int32, C.c_int32, _F, _I32]
        L.orc_kmeans_lloyd.restype = C.c_int32
        _I8 = C.POINTER(C.c_int8)
        L.orc_i8_dot_rows.argtypes = [_I8, _I8, C.c_int64, C.c_int64, _F]
        L.orc_dot_rows_gather.argtypes = [_F, _F, _U32, C.c_int64, C.c_int64, _F]
        L.orc_int8_planes.argtypes = [_F, C.c_int64, C.c_int64, _I8, _F, _F, _F, _F]
        L.orc_bounded_exact_scan.argtypes = [_F, _F, _F, C.c_float, C.c_int64, C.c_int64,
                                             C.c_int32, C.c_int32, C.c_int32, _I8, _F, _F, _F,
                                             _F, C.c_void_p, C.c_void_p, _F, _U32]
        L.orc_bounded_exact_scan.restype = C.c_int
        L.orc_bounded_exact_batch.argtypes = [_F, C.c_int64, _F, _F, _F, C.c_int64, C.c_int64,
                                              C.c_int32, C.c_int32, C.c_int32, C.c_int32, _I8,
                                              _F, _F, _F, _F, C.c_void_p, C.c_void_p, C.c_int32,
                                              _F, _U32, _I32]
        _lib = L
    return _lib


def ref_lib():
    """The reference's own dots.c (None when it was never built here)."""
    global _ref
    if _ref is None:
        path = _build.REF_SO
        if not os.path.exists(path):
            _build.build_reference()
        if not os.path.exists(path):
            return None
        R = C.CDLL(path)
        R.mans_f32_dot_rows.argtypes = [_F, _F, C.c_int64, C.c_int64, _F]
        R.mans_f32_dot_rows_gather.argtypes = [_F, _F, _U32, C.c_int64, C.c_int64, _F]
        R.mans_i8_dot_rows_f32.argtypes = [C.POINTER(C.c_int8), C.POINTER(C.c_int8), C.c_int64,
                                           C.c_int64, _F]
        _ref = R
    return _ref


def ref_dot_rows_ptr():
    """Function pointer of the reference mans_f32_dot_rows, or None."""
    R = ref_lib()
    if R is None:
        return None
    return C.cast(R.mans_f32_dot_rows, C.c_void_p).value


def _p(a, t):
    return a.ctypes.data_as(t)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def lcg_vectors(count, dim, seed):
    out = np.empty((count, dim), np.float32)
    lib().orc_lcg_vectors(seed, count, dim, _p(out, _F))
    return out


def lcg32_vectors(count, dim, seed):
    out = np.empty((count, dim), np.float32)
    lib().orc_lcg32_vectors(seed, count, dim, _p(out, _F))
    return out


def int8_fill(rows):
    """Int8CodeBuffer.fill codes (n x d int8) and per-row scales."""
    rows = f32(rows)
    n, d = rows.shape
    codes = np.empty((n, d), np.int8)
    scales = np.empty(n, np.float32)
    lib().orc_int8_fill(_p(rows, _F), n, d, codes.ctypes.data, _p(scales, _F))
    return codes, scales


def dot_rows(corpus, query, order="seq"):
    corpus, query = f32(corpus), f32(query)
    n, d = corpus.shape
    out = np.empty(n, np.float32)
    fn = lib().orc_dot_rows_seq if order == "seq" else lib().orc_dot_rows_neon
    fn(_p(corpus, _F), _p(query, _F), n, d, _p(out, _F))
    return out


def ref_dot_rows(corpus, query):
    R = ref_lib()
    corpus, query = f32(corpus), f32(query)
    n, d = corpus.shape
    out = np.empty(n, np.float32)
    R.mans_f32_dot_rows(_p(corpus, _F), _p(query, _F), n, d, _p(out, _F))
    return out


def row_norms(corpus):
    corpus = f32(corpus)
    n, d = corpus.shape
    out = np.empty(n, np.float32)
    lib().orc_row_norms(_p(corpus, _F), n, d, _p(out, _F))
    return out


def norm_sq(v):
    v = f32(v)
    return float(lib().orc_norm_sq(_p(v, _F), v.shape[-1]))


def flat_search(corpus, queries, k, metric, norms=None, use_reference_dots=False):
    """Exact (distance, id)-ordered top-k.  Returns (dist[nq,kout], ids, counts)."""
    corpus, queries = f32(corpus), f32(np.atleast_2d(queries))
    n, d = corpus.shape
    nq = queries.shape[0]
    if norms is None and metric in (COSINE, L2):
        norms = row_norms(corpus)
    kout = min(k, MAX_TOPK)
    od = np.empty((nq, kout), np.float32)
    oi = np.empty((nq, kout), np.uint32)
    oc = np.empty(nq, np.int32)
    fn = ref_dot_rows_ptr() if use_reference_dots else None
    npn = None if norms is None else f32(norms)
    lib().orc_flat_search(_p(corpus, _F), None if npn is None else _p(npn, _F), n, d,
                          _p(queries, _F), nq, k, metric, fn, _p(od, _F), _p(oi, _U32), _p(oc, _I32))
    return od, oi, oc


def parallel_flat_scan(corpus, query, k, metric, cores, norms=None, use_reference_dots=True):
    """The reference CPU exact path (ParallelFlatScan) for one query."""
    corpus, query = f32(corpus), f32(query)
    n, d = corpus.shape
    if norms is None and metric in (COSINE, L2):
        norms = row_norms(corpus)
    qn = norm_sq(query) if metric in (COSINE, L2) else 0.0
    od = np.empty(max(1, min(k, n)), np.float32)
    oi = np.empty(max(1, min(k, n)), np.uint32)
    fn = ref_dot_rows_ptr() if use_reference_dots else None
    npn = None if norms is None else f32(norms)
    cnt = lib().orc_parallel_flat_scan(_p(query, _F), _p(corpus, _F),
                                       None if npn is None else _p(npn, _F), qn, n, d, k, metric,
                                       cores, fn, _p(od, _F), _p(oi, _U32))
    return od[:cnt], oi[:cnt]


def gpu_tier_topk(row, k):
    row = f32(row)
    od = np.empty(max(1, k), np.float32)
    oi = np.empty(max(1, k), np.uint32)
    cnt = lib().orc_gpu_tier_topk(_p(row, _F), row.shape[0], k, _p(od, _F), _p(oi, _U32))
    return od[:cnt], oi[:cnt]


def ivf_assign(corpus, centroids, metric):
    corpus, centroids = f32(corpus), f32(centroids)
    n, d = corpus.shape
    nlist = centroids.shape[0]
    rn, cn = row_norms(corpus), row_norms(centroids)
    out = np.empty(n, np.int32)
    lib().orc_ivf_assign(_p(corpus, _F), _p(rn, _F), n, d, _p(centroids, _F), _p(cn, _F), nlist,
                         metric, _p(out, _I32))
    return out


def ivf_layout(corpus, assign, nlist):
    corpus = f32(corpus)
    n, d = corpus.shape
    rn = row_norms(corpus)
    assign = np.ascontiguousarray(assign, np.int32)
    offsets = np.empty(nlist + 1, np.int64)
    ids = np.empty(n, np.uint32)
    packed = np.empty((n, d), np.float32)
    pn = np.empty(n, np.float32)
    lib().orc_ivf_layout(_p(corpus, _F), _p(rn, _F), n, d, _p(assign, _I32), nlist,
                         _p(offsets, _I64), _p(ids, _U32), _p(packed, _F), _p(pn, _F))
    return offsets, ids, packed, pn


def ivf_search(centroids, packed, packed_norms, list_ids, offsets, queries, k, nprobe, metric):
    centroids, packed, queries = f32(centroids), f32(packed), f32(np.atleast_2d(queries))
    packed_norms = f32(packed_norms)
    list_ids = np.ascontiguousarray(list_ids, np.uint32)
    offsets = np.ascontiguousarray(offsets, np.int64)
    nlist, d = centroids.shape
    n = packed.shape[0]
    nq = queries.shape[0]
    cn = row_norms(centroids)
    kout = min(k, MAX_TOPK)
    od = np.empty((nq, max(kout, 0)), np.float32)
    oi = np.empty((nq, max(kout, 0)), np.uint32)
    oc = np.empty(nq, np.int32)
    lib().orc_ivf_search(_p(centroids, _F), _p(cn, _F), nlist, _p(packed, _F), _p(packed_norms, _F),
                         _p(list_ids, _U32), _p(offsets, _I64), n, d, _p(queries, _F), nq, k,
                         nprobe, metric, _p(od, _F), _p(oi, _U32), _p(oc, _I32))
    return od, oi, oc


def simd_distance(a, b, metric):
    a, b = f32(a), f32(b)
    return float(lib().orc_simd_distance(_p(a, _F), _p(b, _F), a.shape[-1], metric))


def pq_lut(query, codebooks, metric):
    """codebooks: [m, ks, sub] float32."""
    query, codebooks = f32(query), f32(codebooks)
    m, ks, sub = codebooks.shape
    out = np.empty((m, ks), np.float32)
    lib().orc_pq_lut(_p(query, _F), _p(codebooks, _F), m, ks, sub, metric, _p(out, _F))
    return out


def pq_encode_subtracting(v, centroid, codebooks):
    v, centroid, codebooks = f32(v), f32(centroid), f32(codebooks)
    m, ks, sub = codebooks.shape
    out = np.empty(m, np.uint8)
    lib().orc_pq_encode_subtracting(_p(v, _F), _p(centroid, _F), _p(codebooks, _F), m, ks, sub,
                                    _p(out, _U8))
    return out


def nearest_coarse(v, coarse, metric):
    v, coarse = f32(v), f32(coarse)
    return int(lib().orc_nearest_coarse(_p(v, _F), _p(coarse, _F), coarse.shape[0],
                                        coarse.shape[1], metric))


def kmeans_lloyd(vectors, centroids, max_iter, metric, workers, offset=0, dim=None):
    """KMeans.cluster's Lloyd iterations (KMeans.swift:95-254) from the given
    initial centroids; rows' sub-vectors [offset, offset + dim).  Returns
    (centroids, assignments, updates)."""
    v = f32(vectors)
    n, stride = v.shape
    dim = stride - offset if dim is None else dim
    cent = np.array(f32(centroids), copy=True)
    k = cent.shape[0]
    assign = np.empty(n, np.int32)
    it = lib().orc_kmeans_lloyd(_p(v, _F), n, stride, offset, dim, k, max_iter, metric, workers,
                                _p(cent, _F), _p(assign, _I32))
    return cent, assign, int(it)


def pq_train_codebooks(vectors, codebooks, max_iter, workers):
    """ProductQuantizer.train's per-subspace clustering (ProductQuantizer.swift
    :10-86: KMeans.clusterSubspace, L2, k = 256) from given initial
    codebooks (m x ks x sub); returns the trained codebooks."""
    v = f32(vectors)
    cb = np.array(f32(codebooks), copy=True)
    m, ks, sub = cb.shape
    for s in range(m):
        cb[s], _, _ = kmeans_lloyd(v, cb[s], max_iter, L2, workers, offset=s * sub, dim=sub)
    return cb


def pq_adc(lut, codes):
    lut = f32(lut)
    m, ks = lut.shape
    codes = np.ascontiguousarray(codes, np.uint8)
    out = np.empty(codes.shape[0], np.float32)
    lib().orc_pq_adc(_p(lut, _F), m, ks, _p(codes, _U8), codes.shape[0], _p(out, _F))
    return out


def ivfpq_search(coarse, codebooks, codes, list_offsets, lists, queries, k, nprobe, metric):
    coarse, codebooks, queries = f32(coarse), f32(codebooks), f32(np.atleast_2d(queries))
    codes = np.ascontiguousarray(codes, np.uint8)
    list_offsets = np.ascontiguousarray(list_offsets, np.int64)
    lists = np.ascontiguousarray(lists, np.uint32)
    nlist, d = coarse.shape
    m, ks, sub = codebooks.shape
    nq = queries.shape[0]
    kout = max(k, 0)  # BoundedSortedList(capacity: k) has no cap beyond k
    od = np.empty((nq, kout), np.float32)
    oi = np.empty((nq, kout), np.uint32)
    oc = np.empty(nq, np.int32)
    lib().orc_ivfpq_search(_p(coarse, _F), nlist, d, _p(codebooks, _F), m, ks, _p(codes, _U8),
                           _p(list_offsets, _I64), _p(lists, _U32), _p(queries, _F), nq, k, nprobe,
                           metric, _p(od, _F), _p(oi, _U32), _p(oc, _I32))
    return od, oi, oc


# ---- BoundedExactScan (the reference's CPU batch route) ---------------------

_I8P = C.POINTER(C.c_int8)


def slice_count(n, cores):
    """ParallelFlatScan.sliceCount: max(1, min(cores, 32, n / 2048))."""
    return max(1, min(cores, 32, n // 2048))


def int8_planes(rows):
    """Int8CodeBuffer.fill: (codes n x d int8, u, w, |v|^2, 1/|v|) planes."""
    rows = f32(rows)
    n, d = rows.shape
    codes = np.empty((n, d), np.int8)
    u, w, nsq, inv = (np.empty(n, np.float32) for _ in range(4))
    lib().orc_int8_planes(_p(rows, _F), n, d, _p(codes, _I8P), _p(u, _F), _p(w, _F),
                          _p(nsq, _F), _p(inv, _F))
    return codes, u, w, nsq, inv


def _ref_bounded_fns(use_reference_dots):
    if not use_reference_dots:
        return None, None
    R = ref_lib()
    if R is None:
        return None, None
    return (C.cast(R.mans_i8_dot_rows_f32, C.c_void_p).value,
            C.cast(R.mans_f32_dot_rows_gather, C.c_void_p).value)


def bounded_exact_batch(corpus, planes, queries, k, metric, threads, cores=None, norms=None,
                        use_reference_dots=True):
    """FlatGPUSearch's CPU batch route at n >= 16384: BoundedExactScan per
    query, queries spread over `threads` workers.  Returns (dist[nq, k'],
    ids, counts) with k' = min(k, n); a count of -1 marks a declined query."""
    corpus, queries = f32(corpus), f32(np.atleast_2d(queries))
    n, d = corpus.shape
    nq = queries.shape[0]
    if norms is None and metric in (COSINE, L2):
        norms = row_norms(corpus)
    qn = (np.array([norm_sq(x) for x in queries], np.float32) if metric in (COSINE, L2)
          else np.zeros(nq, np.float32))
    codes, u, w, nsq, inv = planes
    kout = max(1, min(k, n))
    od = np.full((nq, kout), np.inf, np.float32)
    oi = np.full((nq, kout), 0xFFFFFFFF, np.uint32)
    oc = np.empty(nq, np.int32)
    i8fn, gfn = _ref_bounded_fns(use_reference_dots)
    npn = None if norms is None else f32(norms)
    lib().orc_bounded_exact_batch(
        _p(queries, _F), nq, _p(qn, _F), _p(corpus, _F), None if npn is None else _p(npn, _F),
        n, d, k, metric, slice_count(n, cores or os.cpu_count() or 1), threads,
        _p(codes, _I8P), _p(u, _F), _p(w, _F), _p(nsq, _F), _p(inv, _F), i8fn, gfn, kout,
        _p(od, _F), _p(oi, _U32), _p(oc, _I32))
    return od, oi, oc
