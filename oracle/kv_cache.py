"""Host-KV cache writer oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py)."""
from __future__ import annotations

import numpy as np


def static_cache_update(cache: np.ndarray, states: np.ndarray, cache_position=None) -> int:
    """app/python/pinned_static_cache.py:47-107 (PinnedStaticCache.update and
    _copy_into_cache) for one layer's key or value cache [B, H, S_max, D]:
    token i of ``states`` [B, H, T, D] goes to position cache_position[i]
    (0..T-1 when not given); a later write to a position replaces the earlier
    one.  Returns the cache's sequence length after the update (one past the
    largest position written, 0 for an empty update)."""
    T = states.shape[2]
    pos = np.arange(T) if cache_position is None else np.asarray(cache_position, dtype=np.int64).reshape(-1)
    if pos.shape[0] != T:
        raise ValueError("cache_position length must match key/value sequence length")
    for i, p in enumerate(pos):
        cache[:, :, int(p)] = states[:, :, i]
    return int(pos.max()) + 1 if T else 0


def paged_append(pool_dev, pool_host, block_table: np.ndarray, positions: np.ndarray, new: np.ndarray) -> None:
    """The paged form of the same write, one token per sequence: ``new`` [B, Hkv, D]
    row b goes to page block_table[b, p // page_size] (device page v >= 0, host
    page -1-v < 0), slot p % page_size, with p = positions[b].  Pools are
    [pages, Hkv, page_size, D]."""
    pool = pool_dev if pool_dev is not None else pool_host
    P = pool.shape[2]
    for b, p in enumerate(np.asarray(positions).reshape(-1)):
        e = int(block_table[b, int(p) // P])
        dst = pool_dev[e] if e >= 0 else pool_host[-1 - e]
        dst[:, int(p) % P] = new[b]
