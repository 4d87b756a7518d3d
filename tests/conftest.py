"""pytest configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs on a CPU-only machine (oracle vs golden vectors, host
logic, the C-ABI symbol table, error paths that launch nothing).  ``-m gpu``
tests need an sm_100 GPU and call the CUDA library through its C ABI.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "gemma4-12b-snapdragonx2elite_b200")
for p in (REPO, PKG_ROOT, os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
