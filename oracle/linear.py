"""Offloaded linear oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py)."""
from __future__ import annotations

import numpy as np

TILE_M = 64


def linear(x: np.ndarray, w: np.ndarray, acc=np.float64) -> np.ndarray:
    """y = x @ w.T with w [N_out, K] as nn.Linear stores it, accumulated in
    ``acc`` (the reference's check is nn.Linear, benchmark/benchmark_linear.py:121-123;
    its kernels compute C[N, M] = B[N, K] . A[K, M], include/task/gemv.cuh:267-368)."""
    xa = np.asarray(x, dtype=acc)
    wa = np.asarray(w, dtype=acc)  # no copy when the weights are already stored in `acc`
    return (xa @ wa.T).astype(np.float32, copy=False)


def split_horizontal(m: int, ratio: float, tile_m: int = TILE_M) -> tuple[int, int]:
    """app/python/utils.py:18-45: host rows m_h = floor(m/64 * ratio) * 64."""
    assert m % tile_m == 0
    m_h = int((m // tile_m) * ratio) * tile_m
    return m_h, m - m_h


def horizontal_split(w: np.ndarray, h_m: int, host_side: str = "first") -> tuple[np.ndarray, np.ndarray]:
    """app/python/layers/linearLayer.py:207-246: transposed host slab [K, h_m]
    and device slab [K, d_m]; the reference keeps the first h_m rows on host."""
    n = w.shape[0]
    if host_side == "first":
        return np.ascontiguousarray(w[:h_m].T), np.ascontiguousarray(w[h_m:].T)
    return np.ascontiguousarray(w[n - h_m:].T), np.ascontiguousarray(w[: n - h_m].T)


def gemv_horizontal(wh_t: np.ndarray, wd_t: np.ndarray, x: np.ndarray, host_side: str = "first",
                    acc=np.float64) -> np.ndarray:
    """include/task/gemv.cuh:408-452: output rows [0, h_M) from the host slab and
    [h_M, h_M + d_M) from the device slab (M_offset = h_M, gemv.cuh:438)."""
    xh = x.astype(acc)
    yh = xh @ wh_t.astype(acc)
    yd = xh @ wd_t.astype(acc)
    parts = (yh, yd) if host_side == "first" else (yd, yh)
    return np.concatenate(parts, axis=1).astype(np.float32)
