"""The C ABI library loads and exports every function include/mans_cuda.h
declares (no device calls: runs without a GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", h)).read()
            names += re.findall(r"^\s*(?:int32_t|int64_t|void)\s+(mans_\w+)\s*\(", txt, re.M)
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert "mans_flat_search" in names and "mans_ctx_create" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    from meltan_b200 import _lib
    L = _lib.lib()
    for name in _declared():
        assert hasattr(L, name), name
    assert set(_declared()) == set(_lib.exported_symbols())


def test_no_device_context_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import meltan_b200 as mb
    with pytest.raises(mb.DeviceNotSupported):
        mb.Context(0)


def test_errors_map_to_reference_degradeable_set():
    import meltan_b200 as mb
    assert mb.SearchFailed("x").is_tier_degradeable
    assert mb.GPUExecutionFailed("x").is_tier_degradeable
    assert mb.GPUResourceExhausted("x").is_tier_degradeable
    assert mb.GPUPipelineUnavailable("x").is_tier_degradeable
    assert not mb.DimensionMismatch("x").is_tier_degradeable
    assert not mb.ConstructionFailed("x").is_tier_degradeable
