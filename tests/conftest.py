"""Shared test setup: import paths, the ``gpu`` marker and parity metrics.

GPU tests (``-m gpu``) run on a B200 through the C ABI; everything else runs on
CPU (oracle vs golden vectors, host-side checks, gloo multi-process logic).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "qwen-drive-edge-orin_b200"
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


# ---------------------------------------------------------------- metrics
# The reference harness's parity metrics (kernels/harness/parity_test.py:124-153).
def row_cos_min(a, b):
    a = np.asarray(a, np.float64).reshape(-1, np.asarray(a).shape[-1])
    b = np.asarray(b, np.float64).reshape(-1, np.asarray(b).shape[-1])
    na = np.linalg.norm(a, axis=-1)
    nb = np.linalg.norm(b, axis=-1)
    denom = np.maximum(na * nb, 1e-30)
    cos = (a * b).sum(-1) / denom
    # rows that are zero on both sides count as identical
    cos = np.where((na == 0) & (nb == 0), 1.0, cos)
    return float(cos.min()) if cos.size else 1.0


def max_rel(a, b, floor=0.1):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    if a.size == 0:
        return 0.0
    return float((np.abs(a - b) / np.maximum(np.abs(b), floor)).max())


def tensor_l2_rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a - b))


def max_abs(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max()) if a.size else 0.0


def golden_index():
    return json.loads((GOLDEN / "index.json").read_text())["cases"]


@pytest.fixture(scope="session")
def golden():
    return golden_index()
