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


def test_ep_entry_points_validate_without_gpu():
    """Expert-parallel entry points reject bad shapes, pitches and formats before any CUDA call."""
    lib = pkg()._lib.load()
    # scaled-fp16 partial rows: H fp16 + H / 64 exponents, padded to 16 bytes
    assert lib.ppmoe_ep_partial_pitch(1536) == 3104 and lib.ppmoe_ep_partial_pitch(100) == 0
    assert lib.ppmoe_ep_dispatch_workspace_bytes(4096, 4) > 0 and lib.ppmoe_ep_dispatch_workspace_bytes(10, 9) == 0
    # more than 8 ranks, and experts not divisible by the ranks
    rc = lib.ppmoe_ep_dispatch(16, 16, 10, 1536, 64, 9, 1, 16, 3200, 16, 16, 16, 1 << 20, None)
    assert rc == -2 and b"ranks" in lib.ppmoe_last_error()
    rc = lib.ppmoe_ep_dispatch(16, 16, 10, 1536, 63, 2, 1, 16, 3200, 16, 16, 16, 1 << 20, None)
    assert rc == -2
    # row pitch too small for H activations + E/P gate weights
    rc = lib.ppmoe_ep_dispatch(16, 16, 10, 1536, 64, 2, 1, 16, 3072, 16, 16, 16, 1 << 20, None)
    assert rc == -1 and b"row_pitch" in lib.ppmoe_last_error()
    rc = lib.ppmoe_ep_experts(1024, 10, 3072, 1024, 1536, 32, 96, 0, 1024, 1024, 1 << 20, None)
    assert rc == -1 and b"row_pitch" in lib.ppmoe_last_error()
    rc = lib.ppmoe_ep_experts(1024, 10, 3136, 1024, 1536, 32, 96, 7, 1024, 1024, 1 << 20, None)
    assert rc == -1 and b"partial_format" in lib.ppmoe_last_error()
    rc = lib.ppmoe_ep_combine_f16s(16, 3000, 16, 2, 10, 1536, 16, None)
    assert rc == -2 and b"pitch" in lib.ppmoe_last_error()
    assert lib.ppmoe_ep_combine_f16s(16, 3104, 16, 2, 0, 1536, 16, None) == 0  # nothing to combine
