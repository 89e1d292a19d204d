"""Test set-up: import paths for the product package (ckb200, in cuda-kernels-optimized-for-rtx5090_b200/) and the
oracle, the `gpu` marker, and skipping GPU tests on a machine without CUDA (the CPU suite runs with -m "not gpu")."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "cuda-kernels-optimized-for-rtx5090_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a); runs the kernels")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device here (run with -m gpu on a B200)")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
