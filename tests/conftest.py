"""pytest configuration: the `gpu` marker and import paths.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on
the CPU.  The package directory is ``mini-gpt-inference_b200`` (not a Python
identifier), so its parent is put on sys.path to import ``b200attn``.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (REPO, REPO / "mini-gpt-inference_b200", REPO / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
