"""Shared pytest configuration: the `gpu` marker and helpers for both suites.

`-m "not gpu"` runs on any machine (oracle vs golden vectors, host logic,
C-ABI loading, gloo multi-process logic). `-m gpu` needs a B200 and calls
the CUDA kernels through libpkv.so.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(REPO), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libpkv.so")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> tuple[np.ndarray, dict]:
    data = np.load(GOLDEN / f"{name}.npz")
    return data["out"], json.loads(str(data["meta"]))


# Tolerances on the decode output: fp32 caches 1e-5,
# 16-bit caches 2e-2 max-abs against the reference arithmetic.
ATOL = {"float32": 1e-5, "bfloat16": 2e-2, "float16": 2e-2}
