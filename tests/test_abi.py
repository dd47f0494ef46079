"""The C ABI library loads and exports every symbol include/ppmoe.h declares; host-side
argument validation works without a GPU."""
import ctypes
import os
import re

import pytest

from conftest import ROOT, pkg


def header_symbols():
    src = open(os.path.join(ROOT, "include", "ppmoe.h")).read()
    return sorted(set(re.findall(r"PPMOE_API\s+[\w\s\*]+?\b(ppmoe_\w+)\s*\(", src)))


def test_header_symbols_exported():
    lib = pkg()._lib.load()
    syms = header_symbols()
    assert len(syms) >= 9
    for s in syms:
        assert hasattr(lib, s), s
        assert s in pkg()._lib.SIGNATURES, f"{s} missing from the ctypes signature table"


def test_host_validation_without_gpu():
    L = pkg()._lib
    lib = L.load()
    assert lib.ppmoe_version() >= 100
    assert lib.ppmoe_packed_bytes(1536, 64, 96) >= 3 * 1536 * 6144 * 2 + 1536 * 6144 * 2
    assert lib.ppmoe_packed_bytes(100, 64, 96) == 0  # hidden not a multiple of 64
    assert lib.ppmoe_workspace_bytes(16, 1536, 64, 96) > lib.ppmoe_workspace_bytes(1, 1536, 64, 96)
    # invalid token count and null pointers are rejected before any CUDA call
    rc = lib.ppmoe_decode(None, 0, None, 1536, 64, 96, 0.9, None, None, None, None, None, None, 0, 0, None)
    assert rc == -2 and b"tokens" in lib.ppmoe_last_error()
    rc = lib.ppmoe_decode(None, 1, None, 1536, 64, 96, 0.9, None, None, None, None, None, None, 0, 0, None)
    assert rc == -1
    rc = lib.ppmoe_decode(16, 1, 1024, 1536, 300, 96, 0.9, None, 16, None, None, None, 256, 4096, 0, None)
    assert rc == -2 and b"experts" in lib.ppmoe_last_error()
    rc = lib.ppmoe_pack(None, None, None, None, 1536, 64, 96, None, None)
    assert rc == -1
    with pytest.raises(L.PPMoEError):
        L.call("ppmoe_route_logits", None, 4, 64, 0.9, None, None, None)
