"""Shared test setup: import paths, the `gpu` marker, golden fixtures."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cuda-msst-infer_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libmsst_b200.so")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def golden(name: str):
    z = np.load(os.path.join(GOLDEN, name))
    meta = json.loads(str(z["meta"])) if "meta" in z.files else {}
    return z, meta


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def snr_db(est, ref) -> float:
    ref = np.asarray(ref, np.float64)
    err = np.asarray(est, np.float64) - ref
    return float(10 * np.log10(np.sum(ref * ref) / max(np.sum(err * err), 1e-30)))
