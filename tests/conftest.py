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
