"""Build the CPU checker libraries (test infrastructure only).

* ``oracle/libmans_oracle.so`` -- the C restatement in ``mans_oracle.c``.
* ``oracle/_ref/libmans_ref_dots.so`` -- the reference's own
  ``Sources/MetalANNSC/dots.c`` compiled unmodified from the reference tree
  (only where that tree is present; the built file then travels with the
  repository snapshot and is never committed).

Run ``python oracle/build.py`` or call :func:`build`.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
# The reference tree: MANS_REFERENCE_DIR, else a checkout named "reference"
# beside this repository (absent on machines that only run the prebuilt files).
REF_ROOT = os.environ.get("MANS_REFERENCE_DIR") or os.path.join(
    os.path.dirname(os.path.dirname(HERE)), "reference")
CFLAGS = ["-O2", "-std=c11", "-ffp-contract=off", "-fPIC", "-Wall", "-Wno-unused-function"]

ORACLE_SO = os.path.join(HERE, "libmans_oracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_SO = os.path.join(REF_DIR, "libmans_ref_dots.so")


def _run(cmd):
    subprocess.run(cmd, check=True)


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "mans_oracle.c")
    if force or _stale(ORACLE_SO, [src]):
        _run(["gcc", *CFLAGS, "-shared", "-o", ORACLE_SO, src, "-lpthread", "-lm"])
    return ORACLE_SO


def build_reference(force: bool = False) -> str | None:
    """Compile the reference dots.c as-is; returns None when the tree is absent."""
    src = os.path.join(REF_ROOT, "Sources", "MetalANNSC", "dots.c")
    inc = os.path.join(REF_ROOT, "Sources", "MetalANNSC", "include")
    if not os.path.exists(src):
        return REF_SO if os.path.exists(REF_SO) else None
    os.makedirs(REF_DIR, exist_ok=True)
    if force or _stale(REF_SO, [src]):
        _run(["gcc", *CFLAGS, "-I", inc, "-shared", "-o", REF_SO, src])
    return REF_SO


def build(force: bool = False) -> None:
    build_oracle(force)
    build_reference(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(ORACLE_SO)
    print(REF_SO if os.path.exists(REF_SO) else "(reference dots.c not built)")
