"""ctypes binding of ``libmans_cuda.so`` (declared in ``include/mans_cuda.h``).

Loading fails loudly when the shared library is missing: there is no CPU
fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmans_cuda.so")

_F = C.POINTER(C.c_float)
_U32 = C.POINTER(C.c_uint32)
_I32 = C.POINTER(C.c_int32)
_I64 = C.POINTER(C.c_int64)
_U8 = C.POINTER(C.c_uint8)
_VP = C.c_void_p

# (name, restype, argtypes) for every symbol of include/mans_cuda.h
SIGNATURES = {
    "mans_ctx_create": (C.c_int32, [C.c_int32, C.POINTER(_VP)]),
    "mans_ctx_destroy": (C.c_int32, [_VP]),
    "mans_ctx_create_multi": (C.c_int32, [_VP, C.c_int32, C.POINTER(_VP)]),
    "mans_ctx_device_count": (C.c_int32, [_VP]),
    "mans_last_error_message": (C.c_int32, [C.c_char_p, C.c_size_t]),
    "mans_ctx_sm_count": (C.c_int32, [_VP]),
    "mans_ctx_set_tensor_core_batch": (C.c_int32, [_VP, C.c_int32]),
    "mans_ctx_set_tensor_core_format": (C.c_int32, [_VP, C.c_int32]),
    "mans_corpus_int8_codes": (C.c_int32, [_VP, _VP, _VP]),
    "mans_mann_read_info": (C.c_int32, [C.c_char_p, _VP]),
    "mans_corpus_load_mann": (C.c_int32, [_VP, C.c_char_p, C.c_int32, C.c_int32, _VP]),
    "mans_workspace_last_path": (C.c_int32, [_VP, _VP]),
    "mans_workspace_fallbacks": (C.c_int32, [_VP, _I32]),
    "mans_corpus_create": (C.c_int32, [_VP, _VP, C.c_int64, C.c_int64, C.c_uint32, C.POINTER(_VP)]),
    "mans_corpus_update_rows": (C.c_int32, [_VP, C.c_int64, _VP, C.c_int64]),
    "mans_corpus_destroy": (C.c_int32, [_VP]),
    "mans_corpus_count": (C.c_int64, [_VP]),
    "mans_corpus_dim": (C.c_int64, [_VP]),
    "mans_workspace_create": (C.c_int32, [_VP, C.POINTER(_VP)]),
    "mans_workspace_destroy": (C.c_int32, [_VP]),
    "mans_workspace_check": (C.c_int32, [_VP, _VP]),
    "mans_workspace_set_timing": (C.c_int32, [_VP, C.c_int32]),
    "mans_workspace_stats": (C.c_int32, [_VP, C.POINTER(C.c_double), _I64, _I64]),
    "mans_workspace_stage_times": (C.c_int32, [_VP, C.POINTER(C.c_double), _I64, C.c_int32]),
    "mans_flat_search": (C.c_int32, [_VP, _VP, _VP, C.c_int64, C.c_int64, C.c_int32, C.c_int32,
                                     _VP, _VP, _VP]),
    "mans_flat_search_device": (C.c_int32, [_VP, _VP, _VP, _VP, C.c_int64, C.c_int32, C.c_int32,
                                            _VP, _VP, _VP, _VP]),
    "mans_flat_search_noalloc": (C.c_int32, [_VP, _VP, _VP, C.c_int64, C.c_int32, C.c_int32,
                                             _VP, _VP, _VP, _VP]),
    "mans_topk_merge_device": (C.c_int32, [_VP, _VP, _VP, _VP, _VP, C.c_int32, C.c_int64,
                                           C.c_int64, C.c_int32, C.c_int32, _VP, _VP, _VP,
                                           _VP]),
    "mans_exchange_create": (C.c_int32, [_VP, C.c_int32, C.c_int32, C.c_int64, _VP]),
    "mans_exchange_handle": (C.c_int32, [_VP, _VP]),
    "mans_exchange_open": (C.c_int32, [_VP, _VP]),
    "mans_exchange_allgather": (C.c_int32, [_VP, _VP, _VP, C.c_int64, C.c_int32, C.c_int32, _VP,
                                            _VP, _VP, _VP]),
    "mans_exchange_destroy": (C.c_int32, [_VP]),
    "mans_ivf_create": (C.c_int32, [_VP, _VP, C.c_int32, C.c_int64, _VP, _VP, _VP, C.c_int64,
                                    C.POINTER(_VP)]),
    "mans_ivf_destroy": (C.c_int32, [_VP]),
    "mans_ivf_list_count": (C.c_int64, [_VP]),
    "mans_ivf_assign": (C.c_int32, [_VP, _VP, _VP, C.c_int32, C.c_int32, _VP]),
    "mans_ivf_build": (C.c_int32, [_VP, _VP, _VP, C.c_int32, C.c_int32, _VP]),
    "mans_ivf_layout": (C.c_int32, [_VP, _VP, _VP]),
    "mans_ivf_search": (C.c_int32, [_VP, _VP, _VP, C.c_int64, C.c_int64, C.c_int32, C.c_int32,
                                    C.c_int32, _VP, _VP, _VP]),
    "mans_ivf_search_device": (C.c_int32, [_VP, _VP, _VP, _VP, C.c_int64, C.c_int32, C.c_int32,
                                           C.c_int32, _VP, _VP, _VP, _VP]),
    "mans_ivfpq_create": (C.c_int32, [_VP, _VP, C.c_int32, C.c_int64, _VP, C.c_int32, C.c_int32,
                                      _VP, C.c_int64, _VP, _VP, _VP, C.c_int32, C.POINTER(_VP)]),
    "mans_ivfpq_destroy": (C.c_int32, [_VP]),
    "mans_pq_encode": (C.c_int32, [_VP, _VP, C.c_int64, C.c_int64, _VP, C.c_int32, _VP,
                                   C.c_int32, C.c_int32, C.c_int32, _VP, _VP]),
    "mans_ivfpq_search": (C.c_int32, [_VP, _VP, _VP, C.c_int64, C.c_int64, C.c_int32, C.c_int32,
                                      _VP, _VP, _VP]),
    "mans_ivfpq_search_device": (C.c_int32, [_VP, _VP, _VP, _VP, C.c_int64, C.c_int32, C.c_int32,
                                             _VP, _VP, _VP, _VP]),
    "mans_ivfpq_search_partial_device": (C.c_int32, [_VP, _VP, _VP, _VP, C.c_int64, C.c_int32,
                                                     C.c_int32, _VP, _VP]),
    "mans_ivfpq_resolve_device": (C.c_int32, [_VP, _VP, _VP, C.c_int32, C.c_int64, C.c_int64,
                                              C.c_int32, _VP, _VP, _VP, _VP]),
    "mans_pq_adc_list": (C.c_int32, [_VP, _VP, C.c_int64, _VP, C.c_int32, C.c_int32, _VP,
                                     C.c_int64, _VP]),
    "mans_build_info": (C.c_int32, [C.c_char_p, C.c_size_t]),
    "mans_kmeans_lloyd": (C.c_int32, [_VP, _VP, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                      C.c_int32, C.c_int32, C.c_int32, C.c_int32, _VP, _VP,
                                      _VP]),
    "mans_pq_train": (C.c_int32, [_VP, _VP, C.c_int64, C.c_int64, C.c_int32, C.c_int32,
                                  C.c_int32, C.c_int32, _VP]),
}

_lib = None


def lib():
    """Load the CUDA library (raises if it was never built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m meltan_b200.build` "
                "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _check_build(L)
        _lib = L
    return _lib


def build_info(L=None) -> str:
    """Digest of the sources the loaded library was built from."""
    buf = C.create_string_buffer(128)
    (L or lib()).mans_build_info(buf, len(buf))
    return buf.value.decode()


def _check_build(L):
    """The library must come from the sources beside it: a stale build is an
    error, never silently used."""
    from . import build as _build
    want = "sha256:" + _build.source_hash()
    got = build_info(L)
    if got != want:
        raise RuntimeError(f"{LIB_PATH} was built from other sources ({got[:19]}..., these "
                           f"are {want[:19]}...): rebuild with `python -m meltan_b200.build`")


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().mans_last_error_message(buf, len(buf))
    return buf.value.decode(errors="replace")


def exported_symbols():
    return list(SIGNATURES)
