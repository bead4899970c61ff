"""`offload.runtime` for B200: the reference's PyTorch-extension API over the C ABI.

Mirrors the pybind module of src/torch_runtime.cu:424-468 name for name:
module attributes NUM_SMS, MAX_COPY_SMS, BUFFER_SLOTS, TILE_N and the
functions set_smem_size, build_tma_desc, tensormap_replace_address, gemv,
gemv_horizontal, gemv_multicast, gemv_horizontal_multicast,
gemv_multicast_prefill, gemv_horizontal_multicast_prefill, flush_l2_cache and
print_device_name.  Launches go on torch's current CUDA stream, never
synchronize and allocate nothing, so they can be captured in CUDA graphs.
Argument errors raise RuntimeError, as TORCH_CHECK does in the reference.

Two additions serve the B200 build: ``linear_split`` (pointer-level split
linear with explicit output offsets) and ``probe_stream_read`` (host-link and
HBM read bandwidth probe).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import LIB, check
from .trace import traced

_C = _lib.constants()

NUM_SMS: int = _C.num_sms
MAX_COPY_SMS: int = _C.max_copy_sms
BUFFER_SLOTS: int = _C.buffer_slots
TILE_N: int = _C.tile_n

# KERNEL_OPCODES (src/torch_runtime.cu:20-27).
GEMV = 0
GEMV_HORIZONTAL = 1
GEMV_MULTICAST = 2
GEMV_HORIZONTAL_MULTICAST = 3
GEMV_MULTICAST_PREFILL = 4
GEMV_HORIZONTAL_MULTICAST_PREFILL = 5

_DTYPES = {
    torch.float16: _lib.DTYPE_F16,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float32: _lib.DTYPE_F32,
    torch.uint8: _lib.DTYPE_U8,
    torch.int32: _lib.DTYPE_I32,
    torch.uint32: _lib.DTYPE_U32,
}


def dak_dtype(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise RuntimeError(f"Unsupported tensor dtype for TMA: {dtype}") from None


_HAS_CUDA = torch.cuda.is_available()


def _stream_ptr() -> int:
    # Without a device the C ABI still validates its arguments, then reports
    # DAK_ERR_NO_DEVICE; stream 0 is never used in that case.
    return torch.cuda.current_stream().cuda_stream if _HAS_CUDA else 0


def _desc_ptr(desc: torch.Tensor, name: str) -> int:
    if not isinstance(desc, torch.Tensor) or desc.dtype != torch.uint8 or desc.numel() < _lib.DESC_BYTES:
        raise RuntimeError(f"{name} must be a descriptor returned by build_tma_desc")
    if desc.is_cuda:
        raise RuntimeError(f"{name} must be the CPU descriptor tensor returned by build_tma_desc")
    return desc.data_ptr()


def set_smem_size(smem_size: int, opcode: int = GEMV) -> int:
    """src/torch_runtime.cu:373-417.  The sm_100a kernels size their own shared
    memory; this validates the opcode and returns ``smem_size``."""
    r = LIB.dak_set_smem_size(int(smem_size), int(opcode))
    if r == 0 and smem_size != 0:
        import sys

        print(f"Kernel set shared memory failed: {LIB.dak_last_error_message().decode()}", file=sys.stderr)
        return int(smem_size)
    return int(r)


def build_tma_desc(base: torch.Tensor, shape, strides_bytes, box_dim, elem_strides, swizzle_bytes: int) -> torch.Tensor:
    """src/torch_runtime.cu:120-191: descriptor of ``base`` as a CPU uint8 tensor."""
    if base is None or not isinstance(base, torch.Tensor):
        raise RuntimeError("base must be defined")
    if base.numel() <= 0:
        raise RuntimeError("base must have storage")
    shape, strides_bytes, box_dim, elem_strides = (list(v) for v in (shape, strides_bytes, box_dim, elem_strides))
    if len(shape) != len(strides_bytes) + 1:
        raise RuntimeError("shape and strides_bytes must have same length")
    if len(shape) != len(box_dim):
        raise RuntimeError("shape and box_dim must have same length")
    if len(shape) != len(elem_strides):
        raise RuntimeError("shape and elem_strides must have same length")
    desc = torch.empty(_lib.DESC_BYTES, dtype=torch.uint8)
    st = LIB.dak_build_tma_desc(
        desc.data_ptr(), base.data_ptr(), dak_dtype(base.dtype), len(shape),
        _lib.i64_array(shape), _lib.i64_array(strides_bytes), _lib.i64_array(box_dim),
        _lib.i64_array(elem_strides), int(swizzle_bytes),
    )
    check(st, "build_tma_desc")
    return desc


def tensormap_replace_address(desc: torch.Tensor, data: torch.Tensor) -> None:
    """src/torch_runtime.cu:193-198."""
    check(LIB.dak_tensormap_replace_address(_desc_ptr(desc, "desc"), data.data_ptr()), "tensormap_replace_address")


@traced
def gemv(a_desc, b_desc, c_desc, M: int, N: int, K: int, num_copy_blocks: int, smem_size: int, sms_per_row: int) -> None:
    """src/torch_runtime.cu:201-221: C[N, M] = B[N, K] @ A[K, M]."""
    check(LIB.dak_gemv(_desc_ptr(a_desc, "a_desc"), _desc_ptr(b_desc, "b_desc"), _desc_ptr(c_desc, "c_desc"),
                       M, N, K, num_copy_blocks, smem_size, sms_per_row, _stream_ptr()), "gemv")


@traced
def gemv_horizontal(a_desc_h, a_desc_d, b_desc, c_desc, h_M: int, d_M: int, N: int, K: int,
                    num_copy_blocks: int, num_copy_host_blocks: int, smem_size: int,
                    h_sms_per_row: int, d_sms_per_row: int) -> None:
    """src/torch_runtime.cu:223-244: host rows -> C[:, :h_M], device rows -> C[:, h_M:]."""
    check(LIB.dak_gemv_horizontal(
        _desc_ptr(a_desc_h, "a_desc_h") if h_M > 0 else None, _desc_ptr(a_desc_d, "a_desc_d") if d_M > 0 else None,
        _desc_ptr(b_desc, "b_desc"), _desc_ptr(c_desc, "c_desc"), h_M, d_M, N, K, num_copy_blocks,
        num_copy_host_blocks, smem_size, h_sms_per_row, d_sms_per_row, _stream_ptr()), "gemv_horizontal")


@traced
def gemv_multicast(a_desc, b_desc, c_desc, M, N, K, num_copy_blocks, smem_size, sms_per_row) -> None:
    """src/torch_runtime.cu:313-336 (served by the tcgen05 kernel, no multicast)."""
    check(LIB.dak_gemv_multicast(_desc_ptr(a_desc, "a_desc"), _desc_ptr(b_desc, "b_desc"), _desc_ptr(c_desc, "c_desc"),
                                 M, N, K, num_copy_blocks, smem_size, sms_per_row, _stream_ptr()), "gemv_multicast")


@traced
def gemv_multicast_prefill(a_desc, b_desc, c_desc, M, N, K, num_copy_blocks, smem_size, sms_per_row) -> None:
    """src/torch_runtime.cu:338-361."""
    check(LIB.dak_gemv_multicast_prefill(_desc_ptr(a_desc, "a_desc"), _desc_ptr(b_desc, "b_desc"),
                                         _desc_ptr(c_desc, "c_desc"), M, N, K, num_copy_blocks, smem_size,
                                         sms_per_row, _stream_ptr()), "gemv_multicast_prefill")


@traced
def gemv_horizontal_multicast(h_a_desc, d_a_desc, b_desc, c_desc, h_M, d_M, N, K, num_copy_blocks,
                              num_copy_host_blocks, smem_size, h_sms_per_row, d_sms_per_row) -> None:
    """src/torch_runtime.cu:247-278."""
    check(LIB.dak_gemv_horizontal_multicast(
        _desc_ptr(h_a_desc, "h_a_desc") if h_M > 0 else None, _desc_ptr(d_a_desc, "d_a_desc") if d_M > 0 else None,
        _desc_ptr(b_desc, "b_desc"), _desc_ptr(c_desc, "c_desc"), h_M, d_M, N, K, num_copy_blocks,
        num_copy_host_blocks, smem_size, h_sms_per_row, d_sms_per_row, _stream_ptr()), "gemv_horizontal_multicast")


@traced
def gemv_horizontal_multicast_prefill(h_a_desc, d_a_desc, b_desc, c_desc, h_M, d_M, N, K, num_copy_blocks,
                                      num_copy_host_blocks, smem_size, h_sms_per_row, d_sms_per_row) -> None:
    """src/torch_runtime.cu:280-311."""
    check(LIB.dak_gemv_horizontal_multicast_prefill(
        _desc_ptr(h_a_desc, "h_a_desc") if h_M > 0 else None, _desc_ptr(d_a_desc, "d_a_desc") if d_M > 0 else None,
        _desc_ptr(b_desc, "b_desc"), _desc_ptr(c_desc, "c_desc"), h_M, d_M, N, K, num_copy_blocks,
        num_copy_host_blocks, smem_size, h_sms_per_row, d_sms_per_row, _stream_ptr()),
        "gemv_horizontal_multicast_prefill")


def flush_l2_cache(dummy: torch.Tensor, sink: torch.Tensor) -> None:
    """src/torch_runtime.cu:363-371: read ``dummy`` through L2 on the current stream."""
    if dummy.dtype != torch.float32 or sink.dtype != torch.float32:
        raise RuntimeError("dummy and sink must be float32 CUDA tensors")
    check(LIB.dak_flush_l2_cache(dummy.data_ptr(), dummy.numel(), sink.data_ptr(), _stream_ptr()), "flush_l2_cache")


def print_device_name(device_id: int) -> None:
    """src/runtime.cu:9-16."""
    check(LIB.dak_print_device_name(int(device_id)), "print_device_name")


# --------------------------------------------------------------- B200 additions
def _i64(v) -> int:
    return int(v)


@traced
def linear_split(x: torch.Tensor, y: torch.Tensor, w_host: torch.Tensor | None, w_dev: torch.Tensor | None,
                 host_col_offset: int = 0, dev_col_offset: int | None = None, *, host_ctas: int = 0,
                 dev_ctas: int = 0, host_ksplit: int = 0, dev_ksplit: int = 0, path: int = _lib.PATH_AUTO,
                 allreduce=None, glu: bool = False) -> torch.Tensor:
    """y[:, off:off+cols] = x @ w for each tier, with w the transposed weight [K, cols].

    ``x`` is [ntok, K] (row-major, last dim contiguous), ``y`` [ntok, ldy];
    ``w_host`` lives in pinned host memory, ``w_dev`` in HBM; either may be None.
    With ``allreduce`` (a ``tp.SymmetricAllReduce``), y is summed over the ranks
    of its group inside the same kernel (row-parallel layers).  With ``glu``
    the weight's features alternate 16 gate and 16 up rows and
    y[:, (c // 32) * 16 + c % 16] = silu(gate) * up for the pairs (c, c + 16):
    y has half as many columns (``interleave_gate_up`` builds the layout).
    """
    if x.dim() != 2 or y.dim() != 2 or x.stride(1) != 1 or y.stride(1) != 1:
        raise RuntimeError("x and y must be 2-D with a contiguous last dimension")
    ntok, K = x.shape
    if y.shape[0] != ntok:
        raise RuntimeError("x and y must have the same number of rows")
    a = _lib.LinearArgs()
    hc = 0 if w_host is None else w_host.shape[1]
    dc = 0 if w_dev is None else w_dev.shape[1]
    for w, nm in ((w_host, "w_host"), (w_dev, "w_dev")):
        if w is not None:
            if w.dim() != 2 or w.shape[0] != K or w.stride(1) != 1:
                raise RuntimeError(f"{nm} must be [K, cols] with contiguous columns")
            if w.dtype != x.dtype:
                raise RuntimeError(f"{nm} dtype must match x")
    if dev_col_offset is None:
        dev_col_offset = host_col_offset + hc if host_col_offset == 0 else 0
    a.w_host = w_host.data_ptr() if w_host is not None else None
    a.host_cols, a.ld_host, a.host_col_offset = hc, (w_host.stride(0) if w_host is not None else 0), host_col_offset
    a.w_dev = w_dev.data_ptr() if w_dev is not None else None
    a.dev_cols, a.ld_dev, a.dev_col_offset = dc, (w_dev.stride(0) if w_dev is not None else 0), dev_col_offset
    a.x, a.ldx = x.data_ptr(), x.stride(0)
    a.y, a.ldy = y.data_ptr(), y.stride(0)
    a.ntok, a.K, a.dtype = ntok, K, dak_dtype(x.dtype)
    a.host_ctas, a.dev_ctas, a.host_ksplit, a.dev_ksplit, a.path = host_ctas, dev_ctas, host_ksplit, dev_ksplit, path
    if glu:
        if allreduce is not None:
            raise RuntimeError("a gated linear has no fused all-reduce")
        check(LIB.dak_linear_split_glu(ctypes.byref(a), _stream_ptr()), "linear_split_glu")
    elif allreduce is not None:
        check(LIB.dak_linear_split_allreduce(ctypes.byref(a), ctypes.byref(allreduce.args(y)), _stream_ptr()),
              "linear_split_allreduce")
    else:
        check(LIB.dak_linear_split(ctypes.byref(a), _stream_ptr()), "linear_split")
    return y


GLU_BLOCK = 16  # gate / up rows alternate in blocks of this many features


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[F, K] gate and up weights -> the [2F, K] row order ``linear_split(glu=True)``
    reads: 16 gate rows, the 16 matching up rows, the next 16 gate rows, ...
    F must be a multiple of 16."""
    if gate.shape != up.shape or gate.dim() != 2 or gate.shape[0] % GLU_BLOCK:
        raise RuntimeError(f"gate and up must be equal [F, K] with F a multiple of {GLU_BLOCK}")
    f, k = gate.shape
    return torch.stack([gate.reshape(f // GLU_BLOCK, GLU_BLOCK, k), up.reshape(f // GLU_BLOCK, GLU_BLOCK, k)],
                       1).reshape(2 * f, k)


def probe_stream_read(src: torch.Tensor, ctas: int, stages: int = 4, chunk_bytes: int = 32768,
                      nbytes: int | None = None, sink: torch.Tensor | None = None) -> torch.Tensor:
    """Streams ``src`` (HBM or pinned host memory) through shared memory with
    TMA bulk copies; returns the 1-element int32 checksum tensor it writes
    (``sink`` when given, so a CUDA graph of probes holds only probe launches)."""
    if sink is None:
        sink = torch.zeros(1, dtype=torch.int32, device="cuda")
    elif sink.dtype != torch.int32 or not sink.is_cuda or sink.numel() < 1:
        raise RuntimeError("sink must be an int32 CUDA tensor")
    n = src.numel() * src.element_size() if nbytes is None else int(nbytes)
    check(LIB.dak_probe_stream_read(src.data_ptr(), n, ctas, stages, chunk_bytes, sink.data_ptr(), _stream_ptr()),
          "probe_stream_read")
    return sink


def device_status(clear: bool = True) -> int:
    """Device error word of the kernels' bounded waits (0 = none); synchronizes."""
    return _lib.device_status(clear)
