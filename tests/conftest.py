"""Shared pytest set-up: the ``gpu`` marker and the repository root on ``sys.path``.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on a CPU-only machine.
"""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    # GPU tests that land on a machine without a GPU are skipped, never silently passed on the CPU.
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
