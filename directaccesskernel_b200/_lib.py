"""ctypes binding of libdak_b200.so (the C ABI declared in include/dak_b200.h).

The library is the only compute path of this package: if it is missing or
fails to load, importing this module raises ImportError; there is no CPU or
eager fallback.  Build it with ``python -m directaccesskernel_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("DAK_B200_LIB", Path(__file__).resolve().parent / "libdak_b200.so"))

# Status codes (enum dak_status).
DAK_OK = 0
DAK_ERR_INVALID_ARG = 1
DAK_ERR_UNSUPPORTED = 2
DAK_ERR_CUDA = 3
DAK_ERR_DRIVER = 4
DAK_ERR_TIMEOUT = 5
DAK_ERR_ALIGNMENT = 6
DAK_ERR_NO_DEVICE = 7

# Element types (enum dak_dtype).
DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_F32 = 2
DTYPE_U8 = 3
DTYPE_I32 = 4
DTYPE_U32 = 5

# Linear paths (enum dak_linear_path).
PATH_AUTO = 0
PATH_CUDA_CORE = 1
PATH_TCGEN05 = 2

DESC_BYTES = 128

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_vp = ctypes.c_void_p


class Constants(ctypes.Structure):
    _fields_ = [
        ("num_sms", c_int), ("max_copy_sms", c_int), ("buffer_slots", c_int), ("tile_n", c_int),
        ("tile_m", c_int), ("tile_k", c_int), ("mma_tile_m", c_int), ("mma_max_tokens", c_int),
        ("abi_version", c_int),
    ]


class LinearArgs(ctypes.Structure):
    _fields_ = [
        ("w_host", c_vp), ("host_cols", c_i64), ("ld_host", c_i64), ("host_col_offset", c_i64),
        ("w_dev", c_vp), ("dev_cols", c_i64), ("ld_dev", c_i64), ("dev_col_offset", c_i64),
        ("x", c_vp), ("ldx", c_i64), ("y", c_vp), ("ldy", c_i64),
        ("ntok", c_i64), ("K", c_i64), ("dtype", c_int),
        ("host_ctas", c_int), ("dev_ctas", c_int), ("host_ksplit", c_int), ("dev_ksplit", c_int),
        ("path", c_int),
    ]


class AttnDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("query", c_vp), ("q_stride_b", c_i64), ("q_stride_h", c_i64),
        ("key", c_vp), ("value", c_vp), ("kv_stride_b", c_i64), ("kv_stride_h", c_i64),
        ("key_host", c_vp), ("value_host", c_vp), ("kvh_stride_b", c_i64), ("kvh_stride_h", c_i64),
        ("mask", c_vp), ("mask_stride_b", c_i64),
        ("out", c_vp), ("o_stride_b", c_i64), ("o_stride_h", c_i64),
        ("partial_o", c_vp), ("partial_ml", c_vp),
        ("batch", c_int), ("host_size", c_int), ("num_q_heads", c_int), ("num_kv_heads", c_int),
        ("head_dim", c_int), ("seq_len", c_int), ("split_size", c_int),
        ("scaling", ctypes.c_float), ("dtype", c_int),
    ]


class AttnPagedArgs(ctypes.Structure):
    _fields_ = [
        ("query", c_vp), ("q_stride_b", c_i64), ("q_stride_h", c_i64),
        ("k_pool_dev", c_vp), ("v_pool_dev", c_vp), ("k_pool_host", c_vp), ("v_pool_host", c_vp),
        ("block_table", c_vp), ("bt_stride", c_i64), ("seq_lens", c_vp),
        ("out", c_vp), ("o_stride_b", c_i64), ("o_stride_h", c_i64),
        ("partial_o", c_vp), ("partial_ml", c_vp),
        ("batch", c_int), ("num_q_heads", c_int), ("num_kv_heads", c_int), ("head_dim", c_int),
        ("page_size", c_int), ("max_seq_len", c_int), ("split_size", c_int),
        ("scaling", ctypes.c_float), ("dtype", c_int), ("dev_pages", c_i64), ("host_pages", c_i64),
    ]


class AllReduceArgs(ctypes.Structure):
    _fields_ = [
        ("world", c_int), ("rank", c_int), ("buffers", c_vp * 8), ("flags", c_vp * 8),
        ("slot_elems", c_i64), ("epoch", c_vp), ("done", c_vp), ("timeout_us", c_i64),
        ("own_f32", c_vp), ("mc_f32", c_vp), ("publish_only", c_int),
    ]


class KvAppendArgs(ctypes.Structure):
    _fields_ = [
        ("k_new", c_vp), ("v_new", c_vp), ("new_batch_stride", c_i64), ("new_head_stride", c_i64),
        ("k_pool_dev", c_vp), ("v_pool_dev", c_vp), ("dev_pages", c_i64),
        ("k_pool_host", c_vp), ("v_pool_host", c_vp), ("host_pages", c_i64),
        ("block_table", c_vp), ("table_stride", c_i64), ("max_pages", c_int), ("positions", c_vp),
        ("batch", c_int), ("kv_heads", c_int), ("head_dim", c_int), ("page_size", c_int), ("dtype", c_int),
    ]


# name -> (restype, argtypes); the full list of entry points of include/dak_b200.h.
_I64P = ctypes.POINTER(c_i64)
SIGNATURES = {
    "dak_strerror": (ctypes.c_char_p, [c_int]),
    "dak_last_error_message": (ctypes.c_char_p, []),
    "dak_get_constants": (c_int, [ctypes.POINTER(Constants)]),
    "dak_print_device_name": (c_int, [c_int]),
    "dak_set_smem_size": (ctypes.c_size_t, [ctypes.c_size_t, c_int]),
    "dak_build_tma_desc": (c_int, [c_vp, c_vp, c_int, c_int, _I64P, _I64P, _I64P, _I64P, c_int]),
    "dak_tensormap_replace_address": (c_int, [c_vp, c_vp]),
    "dak_gemv": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "dak_gemv_horizontal": (c_int, [c_vp, c_vp, c_vp, c_vp] + [c_int] * 9 + [c_vp]),
    "dak_gemv_multicast": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "dak_gemv_multicast_prefill": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "dak_gemv_horizontal_multicast": (c_int, [c_vp, c_vp, c_vp, c_vp] + [c_int] * 9 + [c_vp]),
    "dak_gemv_horizontal_multicast_prefill": (c_int, [c_vp, c_vp, c_vp, c_vp] + [c_int] * 9 + [c_vp]),
    "dak_linear_split": (c_int, [ctypes.POINTER(LinearArgs), c_vp]),
    "dak_linear_split_glu": (c_int, [ctypes.POINTER(LinearArgs), c_vp]),
    "dak_flush_l2_cache": (c_int, [c_vp, ctypes.c_size_t, c_vp, c_vp]),
    "dak_attn_decode": (c_int, [ctypes.POINTER(AttnDecodeArgs), c_vp]),
    "dak_attn_decode_paged": (c_int, [ctypes.POINTER(AttnPagedArgs), c_vp]),
    "dak_attn_decode_paged_merged": (c_int, [ctypes.POINTER(AttnPagedArgs), c_vp, c_vp]),
    "dak_kv_append_paged": (c_int, [ctypes.POINTER(KvAppendArgs), c_vp]),
    "dak_rope_kv_append": (c_int, [c_vp, c_i64, c_vp, c_vp, c_int, ctypes.POINTER(KvAppendArgs), c_vp]),
    "dak_linear_split_allreduce": (c_int, [ctypes.POINTER(LinearArgs), ctypes.POINTER(AllReduceArgs), c_vp]),
    "dak_rmsnorm_allreduce": (c_int, [ctypes.POINTER(AllReduceArgs), c_vp, c_vp, c_vp, c_int, c_int, c_i64,
                                      ctypes.c_float, c_int, c_vp]),
    "dak_rmsnorm": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_i64, ctypes.c_float, c_int, c_vp]),
    "dak_rope_qk": (c_int, [c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "dak_silu_mul": (c_int, [c_vp, c_i64, c_vp, c_int, c_int, c_int, c_vp]),
    "dak_attn_decode_noalloc": (c_int, [ctypes.POINTER(AttnDecodeArgs), c_vp]),
    "dak_device_status": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "dak_selftest_wait_timeout": (c_int, [ctypes.c_uint, c_vp]),
    "dak_probe_stream_read": (c_int, [c_vp, ctypes.c_size_t, c_int, c_int, c_int, c_vp, c_vp]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: the sm_100a kernels are not built "
            "(run `python -m directaccesskernel_b200.build`); there is no fallback path"
        )
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as e:
        raise ImportError(f"cannot load {LIB_PATH}: {e}") from e
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


class DakError(RuntimeError):
    """A DAK C-ABI call returned a non-zero status."""

    def __init__(self, status: int, where: str):
        detail = LIB.dak_last_error_message().decode(errors="replace")
        name = LIB.dak_strerror(status).decode()
        super().__init__(f"{where}: {name}" + (f": {detail}" if detail else ""))
        self.status = status


def check(status: int, where: str) -> None:
    if status != DAK_OK:
        raise DakError(status, where)


def constants() -> Constants:
    c = Constants()
    check(LIB.dak_get_constants(ctypes.byref(c)), "dak_get_constants")
    return c


def device_status(clear: bool = True) -> int:
    """Reads the device error word (synchronizes the current device)."""
    v = c_int(0)
    check(LIB.dak_device_status(1 if clear else 0, ctypes.byref(v)), "dak_device_status")
    return v.value


def i64_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (c_i64 * max(1, len(vals)))(*vals)
