"""Split-KV decode attention over host-resident and HBM-resident KV.

Mirrors the reference's `opt_attention` package:
  * ``decode`` has the contract of ``opt_attention._C.decode``
    (opt_attention/csrc/opt_attention_ext.cpp:164-337): rows b < host_size of
    the batch read ``key_host``/``value_host`` (pinned host memory), the others
    read ``key``/``value`` (HBM), one query token per sequence, output
    [B, 1, H, D].  Extensions: key/value may have fewer heads than the query
    (GQA), and the key length need not be a multiple of 64;
  * ``opt_attention_forward`` / ``register`` are the Hugging Face hook of
    opt_attention/opt_attention/interface.py:142-197.  Decode (q_len == 1)
    always runs the sm_100a kernel and raises on inputs it cannot serve; the
    prefill step (q_len > 1) takes the stock transformers attention on the GPU,
    as the reference's hook does.
``decode_paged`` serves KV in page pools (page_size tokens per page) whose
pages are individually placed in HBM or in pinned host memory.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from . import _lib
from ._lib import LIB, check
from .runtime import dak_dtype
from .trace import traced

HEAD_DIM = 128
DEFAULT_SPLIT_SIZE = 256


_HAS_CUDA = torch.cuda.is_available()


def _stream_ptr() -> int:
    # Without a device the C ABI still validates its arguments, then reports
    # DAK_ERR_NO_DEVICE; stream 0 is never used in that case.
    return torch.cuda.current_stream().cuda_stream if _HAS_CUDA else 0


def _check_query(query: torch.Tensor) -> None:
    """opt_attention_ext.cpp:19-27."""
    if not query.is_cuda:
        raise RuntimeError("query must be CUDA")
    if query.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("query must be float16 or bfloat16")
    if query.dim() != 4:
        raise RuntimeError("query must have shape [B, H, 1, D]")
    if query.size(2) != 1:
        raise RuntimeError("decode kernel requires q_len == 1")
    if query.size(3) != HEAD_DIM:
        raise RuntimeError("decode kernel requires head_dim == 128")
    if query.stride(3) != 1:
        raise RuntimeError("query head_dim stride must be 1")


def _check_kv_pair(query, key, value, expected_batch, expected_seq_len, expect_cuda, label) -> None:
    """opt_attention_ext.cpp:29-50 (heads may divide the query heads: GQA)."""
    if key.is_cuda != expect_cuda:
        raise RuntimeError(f"{label} key device is not expected")
    if value.is_cuda != expect_cuda:
        raise RuntimeError(f"{label} value device is not expected")
    if key.dtype != query.dtype:
        raise RuntimeError(f"{label} key dtype must match query dtype")
    if value.dtype != query.dtype:
        raise RuntimeError(f"{label} value dtype must match query dtype")
    if key.dim() != 4:
        raise RuntimeError(f"{label} key must have shape [B, H, S, D]")
    if value.dim() != 4:
        raise RuntimeError(f"{label} value must have shape [B, H, S, D]")
    if key.shape != value.shape:
        raise RuntimeError("key and value shapes must match")
    if key.size(0) != expected_batch:
        raise RuntimeError(f"{label} key batch does not match expected split batch size")
    if key.size(1) <= 0 or query.size(1) % key.size(1) != 0:
        raise RuntimeError(f"{label} key heads must divide query heads")
    if key.size(2) != expected_seq_len:
        raise RuntimeError(f"{label} key seq_len must match expected seq_len")
    if key.size(3) != query.size(3):
        raise RuntimeError(f"{label} key head_dim must match query head_dim")
    if key.stride(3) != 1:
        raise RuntimeError(f"{label} key head_dim stride must be 1")
    if value.stride(3) != 1:
        raise RuntimeError(f"{label} value head_dim stride must be 1")
    if key.stride(2) != HEAD_DIM or value.stride(2) != HEAD_DIM:
        raise RuntimeError(f"{label} requires [B,H,S,D] with S stride == D")
    if not expect_cuda and key.numel() > 0 and not (key.is_pinned() and value.is_pinned()):
        raise RuntimeError(f"{label} key/value must be pinned host memory")


def _check_mask(mask, query, seq_len) -> None:
    """opt_attention_ext.cpp:52-60."""
    if not mask.is_cuda:
        raise RuntimeError("attention_mask must be CUDA")
    if mask.dtype != torch.float32:
        raise RuntimeError("attention_mask must be float32")
    if mask.dim() != 4:
        raise RuntimeError("attention_mask must have shape [B, 1, 1, S]")
    if mask.size(0) != query.size(0):
        raise RuntimeError("attention_mask batch must match query batch")
    if mask.size(1) != 1 or mask.size(2) != 1:
        raise RuntimeError("attention_mask must have singleton head and query dims")
    if mask.size(3) != seq_len:
        raise RuntimeError("attention_mask sequence length must match key sequence length")
    if not (mask.stride(3) == 1 or mask.size(3) == 1):
        raise RuntimeError("attention_mask last dimension must be contiguous")


@traced
def decode(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, key_host: torch.Tensor | None = None,
           value_host: torch.Tensor | None = None, host_size: int = 0, attention_mask: torch.Tensor | None = None,
           scaling: float = 1.0, split_size: int = DEFAULT_SPLIT_SIZE, *, partial_o: torch.Tensor | None = None,
           partial_ml: torch.Tensor | None = None) -> torch.Tensor:
    """opt_attention_ext.cpp:164-319: decode attention over batch-split host/device KV."""
    _check_query(query)
    if split_size <= 0:
        raise RuntimeError("split_size must be positive")
    if split_size % 64 != 0:
        raise RuntimeError("split_size must be a multiple of 64")
    total_batch = query.size(0)
    if not (0 <= host_size <= total_batch):
        raise RuntimeError(f"host_size must be in [0, batch_size], got {host_size} for batch_size={total_batch}")
    gpu_batch = total_batch - host_size
    if key.dim() != 4 or value.dim() != 4:
        raise RuntimeError("key/value must have shape [B, H, S, D]")
    if key.size(0) != gpu_batch:
        raise RuntimeError("key/value GPU batch must equal batch_size - host_size")
    seq_len = key.size(2)
    if gpu_batch == 0 and host_size > 0 and key_host is not None:
        seq_len = key_host.size(2)
    _check_kv_pair(query, key, value, gpu_batch, key.size(2), True, "gpu")
    if host_size > 0:
        if key_host is None:
            raise RuntimeError("key_host is required when host_size > 0")
        if value_host is None:
            raise RuntimeError("value_host is required when host_size > 0")
        if key_host.is_cuda:
            raise RuntimeError("key_host must be host memory")
        if value_host.is_cuda:
            raise RuntimeError("value_host must be host memory")
        _check_kv_pair(query, key_host, value_host, host_size, seq_len, False, "host")
        if gpu_batch > 0 and key_host.size(1) != key.size(1):
            raise RuntimeError("host and gpu KV must have the same number of heads")
    kv_heads = key.size(1) if gpu_batch > 0 else key_host.size(1)
    if seq_len <= 0:
        raise RuntimeError("at least one KV source must be available")
    if attention_mask is not None:
        _check_mask(attention_mask, query, seq_len)

    B, H = query.size(0), query.size(1)
    out = torch.empty((B, 1, H, HEAD_DIM), dtype=query.dtype, device=query.device)
    num_splits = (seq_len + split_size - 1) // split_size
    if num_splits > 1:
        if partial_o is None:
            partial_o = torch.empty((B, H, num_splits, HEAD_DIM), dtype=torch.float32, device=query.device)
        if partial_ml is None:
            partial_ml = torch.empty((B, H, num_splits, 2), dtype=torch.float32, device=query.device)

    a = _lib.AttnDecodeArgs()
    a.query, a.q_stride_b, a.q_stride_h = query.data_ptr(), query.stride(0), query.stride(1)
    if gpu_batch > 0:
        a.key, a.value = key.data_ptr(), value.data_ptr()
        a.kv_stride_b, a.kv_stride_h = key.stride(0), key.stride(1)
        if value.stride(0) != key.stride(0) or value.stride(1) != key.stride(1):
            raise RuntimeError("key and value must share strides")
    if host_size > 0:
        a.key_host, a.value_host = key_host.data_ptr(), value_host.data_ptr()
        a.kvh_stride_b, a.kvh_stride_h = key_host.stride(0), key_host.stride(1)
        if value_host.stride(0) != key_host.stride(0) or value_host.stride(1) != key_host.stride(1):
            raise RuntimeError("key_host and value_host must share strides")
    if attention_mask is not None:
        a.mask, a.mask_stride_b = attention_mask.data_ptr(), attention_mask.stride(0)
    a.out, a.o_stride_b, a.o_stride_h = out.data_ptr(), out.stride(0), out.stride(2)
    if num_splits > 1:
        a.partial_o, a.partial_ml = partial_o.data_ptr(), partial_ml.data_ptr()
    a.batch, a.host_size, a.num_q_heads, a.num_kv_heads = B, host_size, H, kv_heads
    a.head_dim, a.seq_len, a.split_size = HEAD_DIM, seq_len, split_size
    a.scaling, a.dtype = float(scaling), dak_dtype(query.dtype)
    check(LIB.dak_attn_decode(ctypes.byref(a), _stream_ptr()), "decode")
    return out


def uses_tma() -> bool:
    """opt_attention_ext.cpp:336: the sm_100a kernel always loads K/V with TMA."""
    return True


def auto_split_size(batch: int, kv_heads: int, max_seq_len: int, num_sms: int | None = None) -> int:
    """Tokens per split (a multiple of 64) for batch x kv_heads x splits CTAs of one
    per SM: the split that minimises waves x (64-token chunks per CTA + 2), the
    2 standing for a CTA's start-up (barrier set-up, first copies in flight).
    This keeps the last wave full instead of leaving it nearly empty."""
    if num_sms is None:
        from .runtime import NUM_SMS as num_sms
    rows = max(1, batch * kv_heads)
    chunks_total = max(1, math.ceil(max_seq_len / 64))
    best, best_cost = 64 * chunks_total, None
    for chunks in range(1, chunks_total + 1):
        splits = math.ceil(chunks_total / chunks)
        if chunks > 1 and math.ceil(chunks_total / (chunks - 1)) == splits:
            continue  # same split count with fewer chunks per CTA
        waves = math.ceil(rows * splits / num_sms)
        cost = waves * (chunks + 2)
        if best_cost is None or cost < best_cost:
            best, best_cost = 64 * chunks, cost
    return best


@traced
def decode_paged(query: torch.Tensor, k_pool_dev: torch.Tensor | None, v_pool_dev: torch.Tensor | None,
                 k_pool_host: torch.Tensor | None, v_pool_host: torch.Tensor | None, block_table: torch.Tensor,
                 seq_lens: torch.Tensor, scaling: float, split_size: int | None = None, *,
                 out: torch.Tensor | None = None, partial_o: torch.Tensor | None = None,
                 partial_ml: torch.Tensor | None = None, max_seq_len: int | None = None,
                 merge_counters: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention over paged KV; returns [B, Hq, D].

    Pools are [pages, Hkv, page_size, D] (one in HBM, one in pinned host
    memory); ``block_table`` [B, max_pages] int32 on the GPU names page j of
    sequence b as v >= 0 (device page v) or v < 0 (host page -1 - v);
    ``seq_lens`` [B] int32 on the GPU.  With ``merge_counters`` (int32 CUDA,
    B * Hkv entries, zero before the first call and left zero by every call)
    the last split of each (sequence, KV head) merges the splits inside the
    attention kernel instead of a second launch; the result is the same."""
    if query.dim() != 3 or query.size(2) != HEAD_DIM or query.stride(2) != 1:
        raise RuntimeError("query must be [B, Hq, 128] with a contiguous last dimension")
    if query.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("query must be float16 or bfloat16")
    pool = k_pool_dev if k_pool_dev is not None else k_pool_host
    if pool is None:
        raise RuntimeError("no KV pool given")
    for t, nm, on_dev in ((k_pool_dev, "k_pool_dev", True), (v_pool_dev, "v_pool_dev", True),
                          (k_pool_host, "k_pool_host", False), (v_pool_host, "v_pool_host", False)):
        if t is None:
            continue
        if t.dim() != 4 or t.size(3) != HEAD_DIM or not t.is_contiguous():
            raise RuntimeError(f"{nm} must be a contiguous [pages, Hkv, page_size, 128] tensor")
        if t.dtype != query.dtype:
            raise RuntimeError(f"{nm} dtype must match query")
        if t.is_cuda != on_dev:
            raise RuntimeError(f"{nm} is on the wrong device")
        if not on_dev and not t.is_pinned():
            raise RuntimeError(f"{nm} must be pinned host memory")
        if t.size(1) != pool.size(1) or t.size(2) != pool.size(2):
            raise RuntimeError("all pools must share Hkv and page_size")
    if (k_pool_dev is None) != (v_pool_dev is None) or (k_pool_host is None) != (v_pool_host is None):
        raise RuntimeError("K and V pools come in pairs")
    if block_table.dtype != torch.int32 or not block_table.is_cuda or block_table.dim() != 2 or block_table.stride(1) != 1:
        raise RuntimeError("block_table must be an int32 CUDA tensor [B, max_pages]")
    if seq_lens.dtype != torch.int32 or not seq_lens.is_cuda or seq_lens.numel() != query.size(0):
        raise RuntimeError("seq_lens must be an int32 CUDA tensor [B]")
    B, Hq = query.size(0), query.size(1)
    Hkv, page_size = pool.size(1), pool.size(2)
    if max_seq_len is None:
        max_seq_len = block_table.size(1) * page_size
    if split_size is None:
        split_size = auto_split_size(B, Hkv, max_seq_len)
    num_splits = (max_seq_len + split_size - 1) // split_size
    if out is None:
        out = torch.empty((B, Hq, HEAD_DIM), dtype=query.dtype, device=query.device)
    if num_splits > 1:
        if partial_o is None:
            partial_o = torch.empty((B, Hq, num_splits, HEAD_DIM), dtype=torch.float32, device=query.device)
        if partial_ml is None:
            partial_ml = torch.empty((B, Hq, num_splits, 2), dtype=torch.float32, device=query.device)
    a = _lib.AttnPagedArgs()
    a.query, a.q_stride_b, a.q_stride_h = query.data_ptr(), query.stride(0), query.stride(1)
    a.k_pool_dev = k_pool_dev.data_ptr() if k_pool_dev is not None else None
    a.v_pool_dev = v_pool_dev.data_ptr() if v_pool_dev is not None else None
    a.k_pool_host = k_pool_host.data_ptr() if k_pool_host is not None else None
    a.v_pool_host = v_pool_host.data_ptr() if v_pool_host is not None else None
    a.block_table, a.bt_stride, a.seq_lens = block_table.data_ptr(), block_table.stride(0), seq_lens.data_ptr()
    a.out, a.o_stride_b, a.o_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    if num_splits > 1:
        a.partial_o, a.partial_ml = partial_o.data_ptr(), partial_ml.data_ptr()
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = B, Hq, Hkv, HEAD_DIM
    a.page_size, a.max_seq_len, a.split_size = page_size, max_seq_len, split_size
    a.scaling, a.dtype = float(scaling), dak_dtype(query.dtype)
    # Page counts let the kernel bound every table entry (out of range: zeros + error word).
    a.dev_pages = k_pool_dev.size(0) if k_pool_dev is not None else 0
    a.host_pages = k_pool_host.size(0) if k_pool_host is not None else 0
    if merge_counters is not None:
        if merge_counters.dtype != torch.int32 or not merge_counters.is_cuda or merge_counters.numel() < B * Hkv \
                or not merge_counters.is_contiguous():
            raise RuntimeError("merge_counters must be a contiguous int32 CUDA tensor of batch * Hkv entries")
        check(LIB.dak_attn_decode_paged_merged(ctypes.byref(a), merge_counters.data_ptr(), _stream_ptr()),
              "decode_paged")
    else:
        check(LIB.dak_attn_decode_paged(ctypes.byref(a), _stream_ptr()), "decode_paged")
    return out


def _kv_append_args(B: int, Hkv: int, D: int, dtype: torch.dtype, k_pool_dev, v_pool_dev, k_pool_host, v_pool_host,
                    block_table: torch.Tensor, positions: torch.Tensor):
    """Checked KvAppendArgs for the paged pools (the layout of ``decode_paged``)."""
    pool = k_pool_dev if k_pool_dev is not None else k_pool_host
    if pool is None:
        raise RuntimeError("no KV pool given")
    for t, nm, on_dev in ((k_pool_dev, "k_pool_dev", True), (v_pool_dev, "v_pool_dev", True),
                          (k_pool_host, "k_pool_host", False), (v_pool_host, "v_pool_host", False)):
        if t is None:
            continue
        if t.dim() != 4 or t.size(1) != Hkv or t.size(3) != D or not t.is_contiguous() or t.dtype != dtype:
            raise RuntimeError(f"{nm} must be a contiguous [pages, {Hkv}, page_size, {D}] tensor of the KV dtype")
        if t.size(2) != pool.size(2):
            raise RuntimeError("all pools must share page_size")
        if t.is_cuda != on_dev or (not on_dev and not t.is_pinned()):
            raise RuntimeError(f"{nm} must be {'CUDA' if on_dev else 'pinned host'} memory")
    if (k_pool_dev is None) != (v_pool_dev is None) or (k_pool_host is None) != (v_pool_host is None):
        raise RuntimeError("K and V pools come in pairs")
    if block_table.dtype != torch.int32 or not block_table.is_cuda or block_table.dim() != 2 or block_table.stride(1) != 1:
        raise RuntimeError("block_table must be an int32 CUDA tensor [B, max_pages]")
    if positions.dtype != torch.int32 or not positions.is_cuda or positions.numel() != B or not positions.is_contiguous():
        raise RuntimeError("positions must be a contiguous int32 CUDA tensor [B]")
    a = _lib.KvAppendArgs()
    if k_pool_dev is not None:
        a.k_pool_dev, a.v_pool_dev, a.dev_pages = k_pool_dev.data_ptr(), v_pool_dev.data_ptr(), k_pool_dev.size(0)
    if k_pool_host is not None:
        a.k_pool_host, a.v_pool_host, a.host_pages = k_pool_host.data_ptr(), v_pool_host.data_ptr(), k_pool_host.size(0)
    a.block_table, a.table_stride, a.max_pages = block_table.data_ptr(), block_table.stride(0), block_table.size(1)
    a.positions = positions.data_ptr()
    a.batch, a.kv_heads, a.head_dim, a.page_size = B, Hkv, D, pool.size(2)
    a.dtype = dak_dtype(dtype)
    return a


@traced
def kv_append_paged(k_new: torch.Tensor, v_new: torch.Tensor, k_pool_dev: torch.Tensor | None,
                    v_pool_dev: torch.Tensor | None, k_pool_host: torch.Tensor | None,
                    v_pool_host: torch.Tensor | None, block_table: torch.Tensor, positions: torch.Tensor) -> None:
    """Writes k_new/v_new [B, Hkv, D] of one new token per sequence into the paged
    pools (the layout of ``decode_paged``) at ``positions`` [B] (int32, CUDA): device
    pages in HBM, host pages straight into pinned host memory from the GPU.
    Replaces the reference's per-step host-cache update
    (app/python/pinned_static_cache.py:47-107)."""
    if k_new.shape != v_new.shape or k_new.dim() != 3 or k_new.stride(2) != 1 or v_new.stride() != k_new.stride():
        raise RuntimeError("k_new and v_new must be [B, Hkv, D] with equal strides and a contiguous last dimension")
    if k_new.dtype not in (torch.float16, torch.bfloat16) or v_new.dtype != k_new.dtype:
        raise RuntimeError("k_new and v_new must be float16 or bfloat16")
    B, Hkv, D = k_new.shape
    a = _kv_append_args(B, Hkv, D, k_new.dtype, k_pool_dev, v_pool_dev, k_pool_host, v_pool_host, block_table,
                        positions)
    a.k_new, a.v_new = k_new.data_ptr(), v_new.data_ptr()
    a.new_batch_stride, a.new_head_stride = k_new.stride(0), k_new.stride(1)
    check(LIB.dak_kv_append_paged(ctypes.byref(a), _stream_ptr()), "kv_append_paged")


@traced
def rope_kv_append(qkv: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor, q_heads: int, kv_heads: int,
                   head_dim: int, q_out: torch.Tensor, k_pool_dev: torch.Tensor | None, v_pool_dev: torch.Tensor | None,
                   k_pool_host: torch.Tensor | None, v_pool_host: torch.Tensor | None,
                   block_table: torch.Tensor) -> None:
    """One decode step's rotary embedding and KV append in one launch: the q heads
    of ``qkv`` [B, (q_heads + 2 kv_heads) * head_dim] rotated into ``q_out``
    [B, q_heads, head_dim]; the rotated k heads and the v heads written into
    the paged pools at ``positions``, exactly as ``decode_ops.rope_qk`` followed by
    ``kv_append_paged`` would write them."""
    if qkv.dim() != 2 or qkv.stride(1) != 1 or qkv.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("qkv must be a 16-bit [B, (q_heads + 2 kv_heads) * head_dim] tensor, last dim contiguous")
    if not q_out.is_contiguous() or q_out.dtype != qkv.dtype or q_out.numel() != qkv.shape[0] * q_heads * head_dim:
        raise RuntimeError("q_out must be a contiguous [B, q_heads, head_dim] tensor of the qkv dtype")
    if inv_freq.dtype != torch.float32 or not inv_freq.is_cuda or inv_freq.numel() != head_dim // 2:
        raise RuntimeError("inv_freq must be a float32 CUDA tensor of head_dim / 2 entries")
    a = _kv_append_args(qkv.shape[0], kv_heads, head_dim, qkv.dtype, k_pool_dev, v_pool_dev, k_pool_host,
                        v_pool_host, block_table, positions)
    check(LIB.dak_rope_kv_append(qkv.data_ptr(), qkv.stride(0), inv_freq.data_ptr(), q_out.data_ptr(), q_heads,
                                 ctypes.byref(a), _stream_ptr()), "rope_kv_append")


# ------------------------------------------------------------ Hugging Face hook
def _pop_host_kv_kwargs(kwargs: dict):
    """interface.py:22-26."""
    key_host = kwargs.pop("key_host", None)
    value_host = kwargs.pop("value_host", None)
    host_size = int(kwargs.pop("host_size", 0))
    return key_host, value_host, host_size


def _prefill_attention(module, query, key, value, attention_mask, dropout, scaling, key_host=None,
                       value_host=None, host_size=0, **kwargs):
    """Prefill (q_len > 1): host KV rows are brought to the GPU and the stock
    transformers attention runs there, as interface.py:29-68 does."""
    if host_size > 0:
        if key_host is None or value_host is None:
            raise ValueError("key_host/value_host are required when host_size > 0")
        kh = key_host.to(device=query.device, dtype=key.dtype, non_blocking=True)
        vh = value_host.to(device=query.device, dtype=value.dtype, non_blocking=True)
        key = kh if key.shape[0] == 0 else torch.cat((kh, key), dim=0)
        value = vh if value.shape[0] == 0 else torch.cat((vh, value), dim=0)
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling, **kwargs)


@traced
def opt_attention_forward(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          attention_mask: torch.Tensor | None, dropout: float = 0.0, scaling: float | None = None,
                          **kwargs):
    """interface.py:142-189: the registered attention function (returns (out, None))."""
    runtime_kwargs = dict(kwargs)
    key_host, value_host, host_size = _pop_host_kv_kwargs(runtime_kwargs)
    if host_size > 0 and (key_host is None or value_host is None):
        raise ValueError("host_size > 0 requires key_host and value_host")
    scale = 1.0 if scaling is None else float(scaling)
    if query.dim() == 4 and query.shape[2] > 1:
        return _prefill_attention(module, query, key, value, attention_mask, dropout, scale, key_host=key_host,
                                  value_host=value_host, host_size=host_size, **runtime_kwargs)
    if runtime_kwargs.get("output_attentions", False):
        raise NotImplementedError("decode attention does not return attention weights")
    if float(dropout) != 0.0:
        raise NotImplementedError("decode attention does not apply dropout")
    mask = attention_mask
    if mask is not None:
        if mask.dtype == torch.bool:
            mask = torch.where(mask, 0.0, torch.finfo(torch.float32).min).to(torch.float32)
        elif mask.dtype is not torch.float32:
            mask = mask.to(torch.float32)
        seq = key.shape[2] if key.shape[0] > 0 else key_host.shape[2]
        mask = mask[..., :seq]
    split_size = int(os.environ.get("OPT_ATTENTION_SPLIT_SIZE", str(DEFAULT_SPLIT_SIZE)))
    out = decode(query, key, value, key_host, value_host, host_size, mask, scale, split_size)
    return out, None


def register(name: str = "vdcores_opt") -> None:
    """interface.py:192-197: installs the hook into transformers' attention registry."""
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    ALL_ATTENTION_FUNCTIONS.register(name, opt_attention_forward)
    ALL_MASK_ATTENTION_FUNCTIONS.register(name, ALL_MASK_ATTENTION_FUNCTIONS["eager"])
