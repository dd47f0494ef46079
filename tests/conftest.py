"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""
import importlib
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

PKG_NAME = "prune_path_openpangu-embedded-1b_b200"

# output tolerance of the north-star contract: max-abs 2e-2 and
# mean-rel = sum|gpu - ref| / sum|ref| 1e-3 on bf16 outputs (fp32 accumulation)
MAX_ABS = 2e-2
MEAN_REL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """End-to-end mask parity against the literal reference (unstable CPU sort), summed over
    every GPU parity check of the session: tokens, mismatching tokens and their causes."""
    try:
        from gpu_helpers import L2_STATS
    except ImportError:
        return
    if not L2_STATS:
        return
    n = sum(s[1] for s in L2_STATS)
    m = sum(s[2] for s in L2_STATS)
    causes = {}
    for s in L2_STATS:
        for k, v in s[3].items():
            causes[k] = causes.get(k, 0) + v
    terminalreporter.write_line(f"mask parity vs literal reference: {m} of {n} tokens differ "
                                f"({100.0 * m / max(n, 1):.3f}%), all explained: {causes}")
    for what, nt, mm, c in L2_STATS:
        if mm:
            terminalreporter.write_line(f"  {what}: {mm}/{nt} {c}")


def pkg():
    return importlib.import_module(PKG_NAME)


def oracle():
    return importlib.import_module("moe_oracle")


def assert_close_out(got, ref, what=""):
    got = got.float().cpu()
    ref = ref.float().cpu()
    d = (got - ref).abs()
    max_abs = d.max().item() if d.numel() else 0.0
    mean_rel = (d.sum() / ref.abs().sum().clamp_min(1e-30)).item() if d.numel() else 0.0
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, f"{what}: max_abs={max_abs:.3e} mean_rel={mean_rel:.3e}"
    return max_abs, mean_rel


@pytest.fixture(scope="session")
def golden():
    return torch.load(os.path.join(ROOT, "tests", "golden", "golden.pt"))


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
