"""Shared test set-up: the `gpu` marker, import paths, and the built libraries.

Tests marked `gpu` need a B200 and run through the C-ABI library (libfa_attn.so); every other
test runs on the CPU: the oracle against the reference's own known answers, host-side logic, and
that the C-ABI library loads and exports every declared symbol.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fusor-ai_b200")
for path in (ROOT, PKG):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover - torch is part of the image
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
