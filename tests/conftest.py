"""Shared test configuration: the `gpu` marker and small helpers.

`-m "not gpu"` tests run on CPU (oracle vs golden fixtures, host logic, ABI
load/export checks); `-m gpu` tests compare the sm_100a kernels, called through
the C ABI, with the oracle on a B200.
"""
from __future__ import annotations

import contextlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_json(name: str):
    return json.loads((GOLDEN / name).read_text())


def golden_npz(name: str):
    return np.load(GOLDEN / name)


def gen(seed: int, shape, dtype=np.float16, scale: float = 1.0) -> np.ndarray:
    """Same input generator as tests/golden/make_golden.py."""
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(dtype)


def checksum(a: np.ndarray) -> str:
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


@contextlib.contextmanager
def cuda_to(target: str):
    """Sends torch.empty/zeros(device='cuda') to `target` and drops pin_memory,
    so host-side placement logic runs on a machine without a GPU."""
    import torch

    orig = {n: getattr(torch, n) for n in ("empty", "zeros")}

    def wrap(fn):
        def inner(*a, **k):
            if str(k.get("device", "")).startswith("cuda"):
                k["device"] = target
            k.pop("pin_memory", None)
            return fn(*a, **k)

        return inner

    for n, f in orig.items():
        setattr(torch, n, wrap(f))
    try:
        yield
    finally:
        for n, f in orig.items():
            setattr(torch, n, f)


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """Normwise max error: max|got - ref| / max|ref|."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))
