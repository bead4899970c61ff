"""Element-wise steps of a Llama decode layer on the GPU (RMSNorm with a fused
residual add, rotary q/k, SiLU-gated product), one launch each.  They follow
transformers' Llama arithmetic op by op (app/python/llama/vanila_llama.py:
227-400 runs the same ops as separate torch kernels)."""
from __future__ import annotations

import torch

from ._lib import LIB, check
from .runtime import dak_dtype
from .trace import traced


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _check16(*ts):
    for t in ts:
        if t.dtype not in (torch.float16, torch.bfloat16) or not t.is_cuda:
            raise RuntimeError("decode ops take float16/bfloat16 CUDA tensors")
        if t.stride(-1) != 1:
            raise RuntimeError("decode ops need a contiguous last dimension")


@traced
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm of x [rows, cols]; with ``residual``, first x + residual, written back
    into ``residual`` (the running hidden state), then normalised."""
    _check16(x, weight)
    rows, cols = x.shape
    if residual is not None:
        _check16(residual)
        if residual.shape != x.shape or residual.stride() != x.stride():
            raise RuntimeError("residual must match x in shape and strides")
    if weight.numel() != cols or not weight.is_contiguous():
        raise RuntimeError("weight must be a contiguous [cols] tensor")
    if out is None:
        out = torch.empty(rows, cols, dtype=x.dtype, device=x.device)
    rp = residual.data_ptr() if residual is not None else None
    check(LIB.dak_rmsnorm(x.data_ptr(), rp, weight.data_ptr(), out.data_ptr(), rp, rows, cols, x.stride(0),
                          float(eps), dak_dtype(x.dtype), _stream()), "rmsnorm")
    return out


@traced
def rope_qk(qkv: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor, q_heads: int, kv_heads: int,
            head_dim: int, q_out: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor) -> None:
    """Rotary q/k of a fused qkv [B, (q_heads + 2 kv_heads) * head_dim] into q_out
    [B, q_heads, head_dim] and k_out [B, kv_heads, head_dim]; v is copied to v_out."""
    _check16(qkv, q_out, k_out, v_out)
    if positions.dtype != torch.int32 or not positions.is_cuda or inv_freq.dtype != torch.float32:
        raise RuntimeError("positions must be int32 CUDA, inv_freq float32 CUDA")
    if not (q_out.is_contiguous() and k_out.is_contiguous() and v_out.is_contiguous()):
        raise RuntimeError("q_out, k_out and v_out must be contiguous")
    check(LIB.dak_rope_qk(qkv.data_ptr(), qkv.stride(0), positions.data_ptr(), inv_freq.data_ptr(), q_out.data_ptr(),
                          k_out.data_ptr(), v_out.data_ptr(), qkv.shape[0], q_heads, kv_heads, head_dim,
                          dak_dtype(qkv.dtype), _stream()), "rope_qk")


@traced
def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * up for gate_up [rows, 2 * cols] = [gate | up]."""
    _check16(gate_up)
    rows, two = gate_up.shape
    cols = two // 2
    if out is None:
        out = torch.empty(rows, cols, dtype=gate_up.dtype, device=gate_up.device)
    check(LIB.dak_silu_mul(gate_up.data_ptr(), gate_up.stride(0), out.data_ptr(), rows, cols,
                           dak_dtype(gate_up.dtype), _stream()), "silu_mul")
    return out
