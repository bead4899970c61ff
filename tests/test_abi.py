"""The C ABI library loads and exports every entry point of include/dak_b200.h;
host-only entry points (descriptors, constants, argument checks) behave as the
reference's pybind functions do (src/torch_runtime.cu:120-198, 373-417).
No compute call is made here."""
import ctypes
import re

import pytest
import torch

from conftest import REPO


def header_functions():
    text = (REPO / "include" / "dak_b200.h").read_text()
    return sorted(set(re.findall(r"DAK_API\s+[\w\s\*]+?\b(dak_\w+)\s*\(", text)))


def test_library_exports_every_header_function():
    from directaccesskernel_b200 import _lib

    names = header_functions()
    assert len(names) >= 19
    for n in names:
        assert hasattr(_lib.LIB, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_constants():
    from offload import runtime

    assert runtime.NUM_SMS > 0
    assert runtime.TILE_N == 8
    assert runtime.BUFFER_SLOTS >= 2
    assert runtime.MAX_COPY_SMS == runtime.NUM_SMS


def test_strerror_and_status_names():
    from directaccesskernel_b200 import _lib

    assert _lib.LIB.dak_strerror(0) == b"success"
    assert _lib.LIB.dak_strerror(5) == b"device wait timed out"


def test_build_desc_roundtrip_and_replace_address():
    from directaccesskernel_b200 import runtime

    w = torch.zeros(256, 192, dtype=torch.float16)
    d = runtime.build_tma_desc(w, [192, 256], [384], [64, 256], [1, 1], 128)
    assert d.dtype == torch.uint8 and d.numel() == 128 and not d.is_cuda
    ptr = int.from_bytes(bytes(d[8:16].tolist()), "little")
    assert ptr == w.data_ptr()
    w2 = torch.zeros(256, 192, dtype=torch.float16)
    runtime.tensormap_replace_address(d, w2)
    assert int.from_bytes(bytes(d[8:16].tolist()), "little") == w2.data_ptr()


@pytest.mark.parametrize("bad,msg", [
    (dict(strides=[384, 1]), "same length"),
    (dict(box=[64]), "box_dim"),
    (dict(swizzle=48), "swizzle"),
    (dict(shape=[0, 256]), "shape\\[0\\] must be > 0"),
    (dict(strides=[100]), "multiple of 16"),
    (dict(box=[300, 256]), "box_dim\\[0\\] must be <= 256"),
    (dict(box=[128, 256]), "swizzle span"),
])
def test_build_desc_errors(bad, msg):
    from directaccesskernel_b200 import runtime

    w = torch.zeros(256, 192, dtype=torch.float16)
    args = dict(shape=[192, 256], strides=[384], box=[64, 256], es=[1, 1], swizzle=128)
    args.update(bad)
    with pytest.raises(RuntimeError, match=msg):
        runtime.build_tma_desc(w, args["shape"], args["strides"], args["box"], args["es"], args["swizzle"])


def test_build_desc_rejects_dtype_and_empty():
    from directaccesskernel_b200 import runtime

    with pytest.raises(RuntimeError, match="dtype"):
        runtime.build_tma_desc(torch.zeros(4, 8, dtype=torch.float64), [8, 4], [64], [8, 4], [1, 1], 0)
    with pytest.raises(RuntimeError, match="storage"):
        runtime.build_tma_desc(torch.zeros(0, dtype=torch.float16), [8], [], [8], [1], 0)


def test_set_smem_size():
    from directaccesskernel_b200 import runtime

    assert runtime.set_smem_size(112640, runtime.GEMV_HORIZONTAL) == 112640
    # Unsupported opcode: the reference prints and returns 0 (torch_runtime.cu:397-400).
    from directaccesskernel_b200 import _lib

    assert _lib.LIB.dak_set_smem_size(1024, 9) == 0


def test_gemv_rejects_bad_descriptors_without_launch():
    from directaccesskernel_b200 import _lib

    junk = (ctypes.c_uint8 * 128)()
    st = _lib.LIB.dak_gemv(ctypes.addressof(junk), ctypes.addressof(junk), ctypes.addressof(junk), 64, 1, 64,
                           0, 0, 1, None)
    assert st == _lib.DAK_ERR_INVALID_ARG
    assert b"not a DAK descriptor" in _lib.LIB.dak_last_error_message()


def test_gemv_shape_mismatch_is_an_error():
    from directaccesskernel_b200 import runtime
    from directaccesskernel_b200.utils import build_tma_wgmma_k, build_tma_wgmma_mn

    w = torch.zeros(256, 192, dtype=torch.float16)
    x = torch.zeros(2, 256, dtype=torch.float16)
    y = torch.zeros(2, 192, dtype=torch.float16)
    _, a = build_tma_wgmma_mn(w, 64, 256)
    _, b = build_tma_wgmma_k(x, 256, 8)
    _, c = build_tma_wgmma_mn(y, 64, 8)
    with pytest.raises(RuntimeError, match="expected"):
        runtime.gemv(a, b, c, 192, 2, 512, 0, 0, 1)  # K does not match A


def test_linear_split_argument_checks():
    from directaccesskernel_b200 import runtime

    x = torch.zeros(2, 64, dtype=torch.float16)
    y = torch.zeros(2, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        runtime.linear_split(x, y, None, torch.zeros(32, 64, dtype=torch.float16))  # K mismatch
    with pytest.raises(RuntimeError):
        runtime.linear_split(x, y, None, torch.zeros(64, 64, dtype=torch.float32))  # dtype mismatch


def _status(fn, *args):
    from directaccesskernel_b200 import _lib

    st = fn(*args)
    return st, _lib.LIB.dak_last_error_message().decode()


def test_decode_op_argument_checks_fail_before_any_launch():
    """The decode-step entry points reject bad arguments with a status code and
    a message, before touching the device (no GPU here)."""
    from directaccesskernel_b200 import _lib

    L = _lib.LIB
    buf = ctypes.c_void_p(0x10000)  # never dereferenced: every call below fails its checks first
    assert _status(L.dak_rmsnorm, buf, None, buf, buf, None, 4, 64, 64, 1e-5, 99, None)[0] == _lib.DAK_ERR_UNSUPPORTED
    st, msg = _status(L.dak_rmsnorm, None, None, buf, buf, None, 4, 64, 64, 1e-5, _lib.DTYPE_F16, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "rmsnorm" in msg
    st, msg = _status(L.dak_rmsnorm, buf, buf, buf, buf, None, 4, 64, 64, 1e-5, _lib.DTYPE_F16, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "residual" in msg
    st, msg = _status(L.dak_rope_qk, buf, 3 * 128, buf, buf, buf, buf, buf, 2, 1, 1, 127, _lib.DTYPE_F16, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "head_dim" in msg
    st, msg = _status(L.dak_rope_qk, buf, 100, buf, buf, buf, buf, buf, 2, 1, 1, 128, _lib.DTYPE_BF16, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "stride" in msg
    st, msg = _status(L.dak_silu_mul, buf, 100, buf, 4, 64, _lib.DTYPE_F16, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "silu_mul" in msg
    st, msg = _status(L.dak_rmsnorm_allreduce, None, buf, buf, buf, 4, 64, 64, 1e-5, _lib.DTYPE_F16, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "rmsnorm_allreduce" in msg


def test_allreduce_and_kv_append_argument_checks():
    from directaccesskernel_b200 import _lib

    L = _lib.LIB
    ar = _lib.AllReduceArgs()
    ar.world, ar.rank = 9, 0
    lin = _lib.LinearArgs()
    st, msg = _status(L.dak_linear_split_allreduce, ctypes.byref(lin), ctypes.byref(ar), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "world" in msg
    ar.world = 2
    st, msg = _status(L.dak_linear_split_allreduce, ctypes.byref(lin), ctypes.byref(ar), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "required" in msg

    a = _lib.KvAppendArgs()
    a.batch, a.kv_heads, a.head_dim, a.page_size, a.max_pages, a.dtype = 2, 1, 128, 16, 4, _lib.DTYPE_F16
    st, msg = _status(L.dak_kv_append_paged, ctypes.byref(a), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "required" in msg
    a.k_new = a.v_new = a.block_table = a.positions = 0x10000
    a.table_stride = 2
    st, msg = _status(L.dak_kv_append_paged, ctypes.byref(a), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "table_stride" in msg
    a.table_stride = 4
    a.dev_pages = 3  # a page count without pools
    st, msg = _status(L.dak_kv_append_paged, ctypes.byref(a), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "pools" in msg
    a.head_dim = 12
    st, msg = _status(L.dak_kv_append_paged, ctypes.byref(a), None)
    assert st == _lib.DAK_ERR_ALIGNMENT and "head_dim" in msg
    a.dtype = _lib.DTYPE_F32
    assert _status(L.dak_kv_append_paged, ctypes.byref(a), None)[0] == _lib.DAK_ERR_UNSUPPORTED


def test_rope_kv_append_argument_checks():
    """The fused rotary + KV append shares the append's pool checks (k_new / v_new
    are not required) and checks its own qkv arguments, before any launch."""
    from directaccesskernel_b200 import _lib

    L = _lib.LIB
    buf = 0x10000
    a = _lib.KvAppendArgs()
    a.batch, a.kv_heads, a.head_dim, a.page_size, a.max_pages, a.dtype = 2, 1, 128, 16, 4, _lib.DTYPE_F16
    st, msg = _status(L.dak_rope_kv_append, buf, 1280, buf, buf, 8, ctypes.byref(a), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "block_table and positions" in msg
    a.block_table = a.positions = buf
    a.table_stride = 4
    st, msg = _status(L.dak_rope_kv_append, buf, 1280, buf, buf, 8, ctypes.byref(a), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "no KV pool" in msg
    st, msg = _status(L.dak_rope_kv_append, buf, 1280, buf, buf, 8, None, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "null" in msg


def test_gated_linear_argument_checks():
    """The gated linear needs 32-feature multiples and room for half the
    features in y; both are checked before any launch."""
    from directaccesskernel_b200 import _lib

    L = _lib.LIB
    a = _lib.LinearArgs()
    a.x = a.y = a.w_dev = 0x10000
    a.ldx, a.K, a.ntok, a.dtype = 64, 64, 4, _lib.DTYPE_F16
    a.dev_cols, a.ld_dev, a.ldy = 48, 48, 24
    st, msg = _status(L.dak_linear_split_glu, ctypes.byref(a), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "multiples of 32" in msg
    a.dev_cols, a.ld_dev, a.ldy = 64, 64, 24
    st, msg = _status(L.dak_linear_split_glu, ctypes.byref(a), None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "outside y" in msg


def test_paged_merged_argument_checks():
    """The in-kernel-merge entry point needs its counter array, and then checks
    its arguments as dak_attn_decode_paged does, before any launch."""
    from directaccesskernel_b200 import _lib

    L = _lib.LIB
    a = _lib.AttnPagedArgs()
    st, msg = _status(L.dak_attn_decode_paged_merged, ctypes.byref(a), None, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "merge_counters is null" in msg
    st, msg = _status(L.dak_attn_decode_paged_merged, None, 0x10000, None)
    assert st == _lib.DAK_ERR_INVALID_ARG and "args is null" in msg
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim, a.split_size, a.dtype = 2, 8, 2, 128, 64, _lib.DTYPE_F16
    a.page_size, a.max_seq_len = 48, 256
    st, msg = _status(L.dak_attn_decode_paged_merged, ctypes.byref(a), 0x10000, None)
    assert st == _lib.DAK_ERR_UNSUPPORTED and "page_size" in msg


STRUCTS = {"Constants": "dak_constants", "LinearArgs": "dak_linear_args", "AllReduceArgs": "dak_allreduce_args",
           "AttnDecodeArgs": "dak_attn_decode_args", "AttnPagedArgs": "dak_attn_paged_args",
           "KvAppendArgs": "dak_kv_append_args"}


def test_struct_layouts_match_the_header(tmp_path):
    """Every ctypes mirror of an argument struct has the size and field offsets
    that a C compiler gives the struct of include/dak_b200.h."""
    import shutil
    import subprocess

    from directaccesskernel_b200 import _lib

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "dak_b200.h"', "int main(void) {"]
    for py, c in STRUCTS.items():
        lines.append(f'  printf("{py} size %zu\\n", sizeof({c}));')
        for name, *_ in getattr(_lib, py)._fields_:
            lines.append(f'  printf("{py} {name} %zu\\n", offsetof({c}, {name}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(REPO / "include"), "-o", str(exe), str(src)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        py, name, val = line.split()
        got[(py, name)] = int(val)
    for py in STRUCTS:
        cls = getattr(_lib, py)
        assert got[(py, "size")] == ctypes.sizeof(cls), py
        for name, *_ in cls._fields_:
            assert got[(py, name)] == getattr(cls, name).offset, (py, name)
