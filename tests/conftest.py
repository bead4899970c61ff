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


def kv_cache_updates():
    """The update sequence of tests/golden/kv_cache.npz (make_golden.py, KV_UPDATES):
    (positions, seed) per update: a 20-token prefill, ten single-token decode
    steps, one scattered 3-token update; K from ``seed``, V from ``seed + 1000``."""
    return [(list(range(20)), 500)] + [([t], 501 + t) for t in range(20, 30)] + [([35, 31, 33], 540)]


# Positions the sequence above writes (the others keep their initial contents).
KV_WRITTEN = sorted(set(range(30)) | {31, 33, 35})


def kv_page_table(batch: int, pages: int) -> np.ndarray:
    """Block table alternating device (v >= 0) and host (-1-v) pages, shifted per sequence."""
    return np.array([[(b * pages + j) if (b + j) % 2 else -1 - (b * pages + j) for j in range(pages)]
                     for b in range(batch)])


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
