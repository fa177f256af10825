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


def test_plain_c_client_compiles_links_and_runs(tmp_path):
    """The header is plain C: a C11 client that takes the address of every
    declared entry point compiles warning-free with gcc, links against
    libmans_cuda.so and, without a GPU, gets MANS_ERR_DEVICE and a message
    from mans_ctx_create -- what a cgo / Swift / ctypes binding relies on."""
    import shutil
    import subprocess

    import torch
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    names = _declared()
    src = tmp_path / "client.c"
    src.write_text(
        '#include <stdio.h>\n#include <string.h>\n#include "mans_cuda.h"\n'
        "typedef void (*fnp)(void);\n"
        "static fnp entry_points[] = {\n"
        + "".join(f"    (fnp){n},\n" for n in names)
        + "};\n"
        "int main(void) {\n"
        "    for (size_t i = 0; i < sizeof entry_points / sizeof entry_points[0]; ++i)\n"
        "        if (!entry_points[i]) return 10;\n"
        "    mans_ctx *ctx = NULL;\n"
        "    int32_t rc = mans_ctx_create(0, &ctx);\n"
        "    char msg[256] = {0};\n"
        "    mans_last_error_message(msg, sizeof msg);\n"
        '    printf("%d %s\\n", (int)rc, msg);\n'
        "    if (rc == MANS_OK) { mans_ctx_destroy(ctx); return 0; }\n"
        "    return rc == MANS_ERR_DEVICE && strlen(msg) > 0 ? 0 : 11;\n"
        "}\n")
    lib_dir = os.path.join(ROOT, "meltan_b200")
    exe = tmp_path / "client"
    cc = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-Wno-cast-function-type",
                         "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                         "-L", lib_dir, "-lmans_cuda", f"-Wl,-rpath,{lib_dir}"],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    if not torch.cuda.is_available():
        assert run.stdout.startswith("7 "), run.stdout  # MANS_ERR_DEVICE
