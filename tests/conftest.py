"""pytest configuration: the ``gpu`` marker and shared fixtures.

Tests marked ``gpu`` need a B200 (sm_100) and the built libparallel_serve.so;
everything else runs on CPU. Inputs are generated with a CPU torch generator
and copied to the device, so CPU oracle and GPU kernels see identical bits.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def cpu_randn(shape, seed, scale=1.0, dtype=torch.float16):
    g = torch.Generator("cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * scale).to(dtype)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu", torch.float64).numpy()


def rel_err(out, ref) -> float:
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(out - ref).max() / (np.abs(ref).mean() + 1e-9))
