"""Test configuration: import paths and the ``gpu`` marker.

``-m gpu`` tests need a B200 and run the CUDA path through the C ABI;
everything else runs on CPU (oracle vs golden vectors, host logic, loading
and symbol checks of the native library, gloo multi-process tests).
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROJECT = os.path.join(REPO, "kimi26-h100-rmsnorm-swiglu-fusion_b200")
for p in (PROJECT, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
