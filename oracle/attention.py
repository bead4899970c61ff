"""Split-KV decode attention oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py)."""
from __future__ import annotations

import numpy as np


def _repeat_kv(k: np.ndarray, n_rep: int) -> np.ndarray:
    """app/python/llama/vanila_llama.py:212-224 (repeat_kv): kv head j serves
    query heads j*n_rep .. j*n_rep + n_rep - 1."""
    return k if n_rep == 1 else np.repeat(k, n_rep, axis=1)


def decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray | None = None,
                     scaling: float = 1.0, acc=np.float64) -> np.ndarray:
    """Eager attention of one query token in FP32 or wider: softmax(q.k^T * scaling
    + mask) . v, as the reference's fallback path computes it
    (opt_attention/opt_attention/interface.py:29-68 -> transformers OPT
    eager_attention_forward; GQA per vanila_llama.py:227-246).
    q [B, Hq, 1, D], k/v [B, Hkv, S, D], mask [B, 1, 1, S]; returns [B, 1, Hq, D]."""
    B, Hq, _, D = q.shape
    n_rep = Hq // k.shape[1]
    kk = _repeat_kv(k.astype(acc), n_rep)
    vv = _repeat_kv(v.astype(acc), n_rep)
    s = np.einsum("bhqd,bhsd->bhqs", q.astype(acc), kk) * scaling
    if mask is not None:
        s = s + mask.astype(acc)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    o = np.einsum("bhqs,bhsd->bhqd", p, vv)
    return np.transpose(o, (0, 2, 1, 3)).astype(np.float32)


def decode_attention_grouped(q: np.ndarray, k: np.ndarray, v: np.ndarray, scaling: float = 1.0,
                             acc=np.float32) -> np.ndarray:
    """``decode_attention`` without a mask, computed per GQA group with matrix
    products instead of materialising repeat_kv: query heads j*n_rep ..
    j*n_rep + n_rep - 1 attend to kv head j (vanila_llama.py:212-246).  Same
    result; this is the form the host-core baseline times.
    q [B, Hq, 1, D], k/v [B, Hkv, S, D]; returns [B, 1, Hq, D]."""
    B, Hq, _, D = q.shape
    Hkv = k.shape[1]
    qg = q.astype(acc, copy=False).reshape(B, Hkv, Hq // Hkv, D)
    kk = k.astype(acc, copy=False)
    s = np.matmul(qg, kk.transpose(0, 1, 3, 2)) * acc(scaling)
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    o = np.matmul(p, v.astype(acc, copy=False))
    return o.reshape(B, 1, Hq, D).astype(np.float32)


def batch_split_decode(q, k_dev, v_dev, k_host, v_host, host_size: int, mask=None, scaling: float = 1.0):
    """`_C.decode` semantics (opt_attention_ext.cpp:164-319; kernel.cuh:331-348):
    rows b < host_size read the host KV, the rest the device KV (row b - host_size)."""
    parts_k = [a for a in (k_host if host_size > 0 else None, k_dev) if a is not None and a.shape[0] > 0]
    parts_v = [a for a in (v_host if host_size > 0 else None, v_dev) if a is not None and a.shape[0] > 0]
    k = np.concatenate(parts_k, axis=0)
    v = np.concatenate(parts_v, axis=0)
    return decode_attention(q, k, v, mask, scaling)


def split_partials(q: np.ndarray, k: np.ndarray, v: np.ndarray, split_size: int, scaling: float = 1.0,
                   mask: np.ndarray | None = None):
    """Per-split partial results of the split-KV pass (kernel.cuh:270-324):
    unnormalised o, running max m and sum l for every (b, head, split).
    q [B, H, D], k/v [B, H, S, D] (heads already matched)."""
    B, H, S, D = k.shape
    ns = (S + split_size - 1) // split_size
    o = np.zeros((B, H, ns, D))
    m = np.full((B, H, ns), -np.inf)
    lsum = np.zeros((B, H, ns))
    for i in range(ns):
        sl = slice(i * split_size, min(S, (i + 1) * split_size))
        s = np.einsum("bhd,bhsd->bhs", q.astype(np.float64), k[:, :, sl].astype(np.float64)) * scaling
        if mask is not None:
            s = s + mask[:, None, sl].astype(np.float64)
        mi = s.max(axis=-1)
        p = np.exp(s - mi[..., None])
        o[:, :, i] = np.einsum("bhs,bhsd->bhd", p, v[:, :, sl].astype(np.float64))
        m[:, :, i] = mi
        lsum[:, :, i] = p.sum(axis=-1)
    return o, m, lsum


def lse_merge(o: np.ndarray, m: np.ndarray, lsum: np.ndarray) -> np.ndarray:
    """opt_attention_reduce_splits_kernel (kernel.cuh:362-386):
    out = sum_i o_i e^(m_i - m*) / sum_i l_i e^(m_i - m*), m* = max_i m_i."""
    gm = m.max(axis=-1, keepdims=True)
    sc = np.where(np.isfinite(m), np.exp(m - gm), 0.0)
    den = (lsum * sc).sum(axis=-1)
    num = (o * sc[..., None]).sum(axis=-2)
    return np.where(den[..., None] == 0, 0.0, num / np.where(den[..., None] == 0, 1.0, den[..., None]))


def paged_gather(pool_dev, pool_host, block_table_row, seq_len: int) -> np.ndarray:
    """Contiguous [Hkv, seq_len, D] view of one sequence from the two page pools
    ([pages, Hkv, page_size, D]); entry v >= 0 is device page v, v < 0 host page -1-v."""
    pool = pool_dev if pool_dev is not None else pool_host
    P = pool.shape[2]
    npages = (seq_len + P - 1) // P
    pages = []
    for j in range(npages):
        e = int(block_table_row[j])
        pages.append(pool_dev[e] if e >= 0 else pool_host[-1 - e])
    kv = np.concatenate(pages, axis=1)  # [Hkv, npages*P, D]
    return kv[:, :seq_len]


def paged_decode(q, k_dev, v_dev, k_host, v_host, block_table, seq_lens, scaling: float) -> np.ndarray:
    """Decode attention of q [B, Hq, D] over paged KV; returns [B, Hq, D]."""
    out = []
    for b in range(q.shape[0]):
        k = paged_gather(k_dev, k_host, block_table[b], int(seq_lens[b]))[None]
        v = paged_gather(v_dev, v_host, block_table[b], int(seq_lens[b]))[None]
        out.append(decode_attention(q[b][None, :, None, :], k, v, None, scaling)[0, 0])
    return np.stack(out)
