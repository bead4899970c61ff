"""Split arithmetic and descriptor helpers, mirroring app/python/utils.py:1-145.

``split_horizontal`` and the two descriptor builders produce exactly the
arguments the reference produces (tests/golden/ pins them against the
reference's own functions); the descriptors they return are this build's
opaque blobs, from which the C ABI rebuilds its sm_100a tile maps.
"""
from __future__ import annotations

import torch

from . import runtime
from .config import (BUFFER_SLOTS, BUFFER_SLOTS_B_MULTICAST, BUFFER_SLOTS_MULTICAST, TILE_K, TILE_K_MULTICAST,
                     TILE_M, TILE_M_MULTICAST, TILE_N, TILE_N_MULTICAST)


def get_smem_size(multicast: bool = False) -> int:
    """app/python/utils.py:7-11 (the value is passed through and not used by the sm_100a kernels)."""
    if not multicast:
        return ((TILE_M * TILE_K + TILE_N * TILE_K) * BUFFER_SLOTS + TILE_M * TILE_N) * 2 + 1024
    return (2 * TILE_M_MULTICAST * TILE_K_MULTICAST * BUFFER_SLOTS_MULTICAST
            + TILE_N_MULTICAST * TILE_K_MULTICAST * BUFFER_SLOTS_B_MULTICAST
            + 2 * TILE_M_MULTICAST * TILE_N_MULTICAST) * 2 + 1024


def get_other_dims(dim: int, i: int):
    """app/python/utils.py:15-16: dims other than ``i`` and the last one."""
    return [j for j in range(dim - 1) if j != i and j - dim != i]


def split_horizontal(weight_shape, offload_ratio):
    """app/python/utils.py:18-45: rows [0, m_h) go to host, m_h = floor(m/64 * r) * 64."""
    m = weight_shape[0]
    assert m % TILE_M == 0, f"Weight shape {weight_shape} is not compatible with tile size {TILE_M}"
    num_tiles = m // TILE_M
    m_h = int(num_tiles * offload_ratio) * TILE_M
    return m_h, m - m_h


def build_tma_wgmma_mn(mat: torch.Tensor, tileM: int, tileK: int, iK: int = -2, debug: bool = False):
    """app/python/utils.py:48-101: descriptor of an MN-major matrix ([K, M], M contiguous)."""
    assert iK != -1 and iK < len(mat.shape) - 1, "iK must not be the last dim"
    assert len(mat.shape) >= 2, "Input matrix must be at least 2D"
    K, M = mat.shape[iK], mat.shape[-1]
    elsize = mat.element_size()
    blockM = 128 // elsize
    blockK = 8
    assert tileM % blockM == 0, f"tileM {tileM} must be multiple of blockM {blockM}"
    if debug:
        global_dims = [blockM, blockK, M // blockM, K // blockK]
        global_strides = [mat.stride(iK), blockM, mat.stride(iK) * blockK]
        box_dims = [blockM, blockK, tileM // blockM, tileK // blockK]
    else:
        global_dims = [M, K]
        global_strides = [mat.stride(iK)]
        box_dims = [tileM, tileK]
    if len(mat.shape) > 2:
        size_otherthan_k_or_m = 1
        other_dims = get_other_dims(len(mat.shape), iK)
        inner_most_others = other_dims[-1]
        for i in other_dims:
            size_otherthan_k_or_m *= mat.shape[i]
        global_dims.append(size_otherthan_k_or_m)
        global_strides.append(mat.stride(inner_most_others))
        box_dims.append(1)
    rank = len(global_dims)
    box_strides = [1] * rank
    global_strides = [s * elsize for s in global_strides]
    return rank, runtime.build_tma_desc(mat, global_dims, global_strides, box_dims, box_strides, 128)


def build_tma_wgmma_k(mat: torch.Tensor, tileK: int, tileN: int, iN: int = -2):
    """app/python/utils.py:104-145: descriptor of a K-major matrix ([N, K], K contiguous)."""
    assert iN != -1 and iN < len(mat.shape) - 1, "iN must not be the last dim"
    N, K = mat.shape[iN], mat.shape[-1]
    elsize = mat.element_size()
    blockK = 128 // elsize
    assert tileK % blockK == 0, "tileK must be multiple of blockK"
    glob_dims = [blockK, N, K // blockK]
    glob_strides = [mat.stride(iN), blockK]
    box_dims = [blockK, tileN, tileK // blockK]
    if len(mat.shape) > 2:
        size_otherthan_k_or_n = 1
        other_dims = get_other_dims(len(mat.shape), iN)
        inner_most_others = other_dims[-1]
        for i in other_dims:
            size_otherthan_k_or_n *= mat.shape[i]
        glob_dims.append(size_otherthan_k_or_n)
        glob_strides.append(mat.stride(inner_most_others))
        box_dims.append(1)
    glob_strides = [s * elsize for s in glob_strides]
    rank = len(glob_dims)
    box_strides = [1] * rank
    return rank, runtime.build_tma_desc(mat, glob_dims, glob_strides, box_dims, box_strides, 128)
