"""dak_attn_decode_noalloc: the allocation-free decode attention entry point.

It serves callers that cannot allocate device memory (a host bound only to the
C ABI without a device allocator, or an engine that has reserved all free
device memory), by keeping the split-KV scratch in a fixed 8 MiB array inside
the library.  These tests call it through the C ABI and compare its output with
the scratch-taking entry point dak_attn_decode on the same inputs, on two calls
in a row, and from a C host that switches CUDA contexts; this file is collected
last so a failure here leaves every other test already run.  The size checks
run before any device work, so they are tested without a GPU."""
import ctypes
import math
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import REPO, rel_err

TOL = 2e-3  # the attention parity tolerance used by the other GPU tests
SCRATCH_FLOATS = 2 << 20  # the library's built-in array: 8 MiB of FP32
CUDA = Path("/usr/local/cuda")
CTX_SRC = REPO / "tests" / "c_abi" / "noalloc_context_check.c"


def _args(q, kd, vd, kh, vh, host, out, split, po=None, pml=None, dtype=None):
    from directaccesskernel_b200 import _lib

    a = _lib.AttnDecodeArgs()
    a.query, a.q_stride_b, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.key, a.value, a.kv_stride_b, a.kv_stride_h = kd.data_ptr(), vd.data_ptr(), kd.stride(0), kd.stride(1)
    if kh is not None:
        a.key_host, a.value_host = kh.data_ptr(), vh.data_ptr()
        a.kvh_stride_b, a.kvh_stride_h = kh.stride(0), kh.stride(1)
    a.out, a.o_stride_b, a.o_stride_h = out.data_ptr(), out.stride(0), out.stride(2)
    if po is not None:
        a.partial_o, a.partial_ml = po.data_ptr(), pml.data_ptr()
    B, H = q.shape[0], q.shape[1]
    a.batch, a.host_size, a.num_q_heads, a.num_kv_heads = B, host, H, kd.shape[1]
    a.head_dim, a.seq_len, a.split_size = 128, kd.shape[2], split
    a.scaling = 1.0 / math.sqrt(128)
    a.dtype = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_F16
    return a


def _inputs(seed, B=4, Hq=8, Hkv=2, S=1000, host=2, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Hq, 1, 128, generator=g) / math.sqrt(128)).to(dtype).cuda()
    k = torch.randn(B, Hkv, S, 128, generator=g).to(dtype)
    v = torch.randn(B, Hkv, S, 128, generator=g).to(dtype)
    if host == 0:
        return q, k.cuda(), v.cuda(), None, None
    return q, k[host:].cuda(), v[host:].cuda(), k[:host].pin_memory(), v[:host].pin_memory()


def _both(seed, split, host, dtype=torch.float16, **shape):
    """Runs dak_attn_decode (caller scratch) and dak_attn_decode_noalloc on the
    same inputs; returns both outputs as FP32 numpy arrays."""
    from directaccesskernel_b200 import _lib

    stream = torch.cuda.current_stream().cuda_stream
    q, kd, vd, kh, vh = _inputs(seed, host=host, dtype=dtype, **shape)
    B, H, S = q.shape[0], q.shape[1], kd.shape[2]
    ns = (S + split - 1) // split
    po = pml = None
    if ns > 1:
        po = torch.empty(B, H, ns, 128, dtype=torch.float32, device="cuda")
        pml = torch.empty(B, H, ns, 2, dtype=torch.float32, device="cuda")
    ref_out = torch.empty(B, 1, H, 128, dtype=dtype, device="cuda")
    got_out = torch.full((B, 1, H, 128), float("nan"), dtype=dtype, device="cuda")
    a = _args(q, kd, vd, kh, vh, host, ref_out, split, po, pml)
    _lib.check(_lib.LIB.dak_attn_decode(ctypes.byref(a), stream), "dak_attn_decode")
    b = _args(q, kd, vd, kh, vh, host, got_out, split)
    _lib.check(_lib.LIB.dak_attn_decode_noalloc(ctypes.byref(b), stream), "dak_attn_decode_noalloc")
    torch.cuda.synchronize()
    got = got_out.float().cpu().numpy()
    assert not np.isnan(got).any()
    return got, ref_out.float().cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("host", [0, 2])
def test_noalloc_matches_scratch_taking_entry_point_on_two_calls(dtype, host):
    from directaccesskernel_b200 import _lib

    for seed in (0, 1):  # two calls in a row; the second reuses the shared array
        got, ref = _both(seed, 64, host, dtype)
        assert rel_err(got, ref) < TOL
    assert _lib.device_status() == 0


@pytest.mark.gpu
def test_noalloc_at_the_edge_of_its_scratch():
    """8 x 32 heads x 63 splits x 130 floats = 2,096,640, 512 floats below the
    array's size: the last partial (m, l) rows sit at the end of the array."""
    from directaccesskernel_b200 import _lib

    B, Hq, split, S = 8, 32, 64, 63 * 64
    assert B * Hq * (S // split) * 130 <= SCRATCH_FLOATS < B * Hq * (S // split + 1) * 130
    for seed in (3, 4):
        got, ref = _both(seed, split, 2, B=B, Hq=Hq, Hkv=8, S=S)
        assert rel_err(got, ref) < TOL
    assert _lib.device_status() == 0


@pytest.mark.gpu
def test_noalloc_single_split_needs_no_scratch():
    """With seq_len <= split_size the output is written directly, so a batch whose
    split partials would not fit the array is still served."""
    from directaccesskernel_b200 import _lib

    B, Hq = 128, 128
    assert B * Hq * 130 > SCRATCH_FLOATS
    got, ref = _both(5, 64, 4, B=B, Hq=Hq, Hkv=16, S=64)
    assert rel_err(got, ref) < TOL
    assert _lib.device_status() == 0


def _reject(batch, q_heads, kv_heads, seq_len, split=64):
    """Calls the entry point with sizes past its scratch; nothing reaches the
    GPU, so the pointers are placeholders."""
    from directaccesskernel_b200 import _lib

    a = _lib.AttnDecodeArgs()
    a.query = a.key = a.value = a.out = 16
    a.batch, a.host_size, a.num_q_heads, a.num_kv_heads = batch, 0, q_heads, kv_heads
    a.head_dim, a.seq_len, a.split_size = 128, seq_len, split
    a.scaling, a.dtype = 1.0, _lib.DTYPE_F16
    return _lib.LIB.dak_attn_decode_noalloc(ctypes.byref(a), None)


def test_noalloc_rejects_calls_beyond_its_scratch():
    from directaccesskernel_b200 import _lib

    assert _reject(64, 64, 8, 1 << 20) == _lib.DAK_ERR_INVALID_ARG  # 64 x 64 x 16384 splits x 130 floats
    assert b"exceeds" in _lib.LIB.dak_last_error_message()
    # One split more than the edge case above.
    assert _reject(8, 32, 8, 64 * 64) == _lib.DAK_ERR_INVALID_ARG
    # Products that would wrap a 64-bit size are rejected, not wrapped.
    assert _reject(1 << 30, 1 << 30, 1 << 27, (1 << 31) - 1) == _lib.DAK_ERR_INVALID_ARG
    assert b"exceeds" in _lib.LIB.dak_last_error_message()


def _build_ctx_check(tmp_path: Path) -> Path:
    cc = shutil.which("gcc")
    if cc is None or not (CUDA / "include" / "cuda.h").exists():
        pytest.skip("no C compiler or CUDA headers")
    lib_dir = REPO / "directaccesskernel_b200"
    if not (lib_dir / "libdak_b200.so").exists():
        pytest.fail("libdak_b200.so is not built")
    exe = tmp_path / "noalloc_context_check"
    # Linked against the driver stub; the real libcuda.so.1 is found at run time.
    subprocess.run([cc, "-O2", "-I", str(REPO / "include"), "-I", str(CUDA / "include"), str(CTX_SRC),
                    "-L", str(lib_dir), "-ldak_b200", "-L", str(CUDA / "lib64" / "stubs"), "-lcuda", "-lm",
                    f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    return exe


def test_context_check_host_compiles_and_links(tmp_path):
    assert _build_ctx_check(tmp_path).exists()


@pytest.mark.gpu
def test_noalloc_follows_the_current_cuda_context(tmp_path):
    """A C host that creates, switches and resets contexts through the driver
    API gets the same output from both entry points in every context."""
    exe = _build_ctx_check(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("ok"), r.stdout
