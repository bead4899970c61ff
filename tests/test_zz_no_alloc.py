"""dak_attn_decode_noalloc: the allocation-free decode attention entry point.

It serves callers that cannot allocate device memory (a host bound only to the
C ABI without a device allocator, or an engine that has reserved all free
device memory), by keeping the split-KV scratch in a fixed 8 MiB array inside
the library.  These tests call it through the C ABI and compare its output with
the scratch-taking entry point dak_attn_decode on the same inputs, on two calls
in a row; this file is collected last so a failure here leaves every other
test already run."""
import ctypes
import math

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 2e-3  # the attention parity tolerance used by the other GPU tests


def _args(q, kd, vd, kh, vh, host, out, split, po=None, pml=None):
    from directaccesskernel_b200 import _lib

    a = _lib.AttnDecodeArgs()
    a.query, a.q_stride_b, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.key, a.value, a.kv_stride_b, a.kv_stride_h = kd.data_ptr(), vd.data_ptr(), kd.stride(0), kd.stride(1)
    a.key_host, a.value_host = kh.data_ptr(), vh.data_ptr()
    a.kvh_stride_b, a.kvh_stride_h = kh.stride(0), kh.stride(1)
    a.out, a.o_stride_b, a.o_stride_h = out.data_ptr(), out.stride(0), out.stride(2)
    if po is not None:
        a.partial_o, a.partial_ml = po.data_ptr(), pml.data_ptr()
    B, H = q.shape[0], q.shape[1]
    a.batch, a.host_size, a.num_q_heads, a.num_kv_heads = B, host, H, kd.shape[1]
    a.head_dim, a.seq_len, a.split_size = 128, kd.shape[2], split
    a.scaling, a.dtype = 1.0 / math.sqrt(128), _lib.DTYPE_F16
    return a


def _inputs(seed, B=4, Hq=8, Hkv=2, S=1000, host=2):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Hq, 1, 128, generator=g) / math.sqrt(128)).half().cuda()
    k = torch.randn(B, Hkv, S, 128, generator=g).half()
    v = torch.randn(B, Hkv, S, 128, generator=g).half()
    return q, k[host:].cuda(), v[host:].cuda(), k[:host].pin_memory(), v[:host].pin_memory()


def test_noalloc_matches_scratch_taking_entry_point_on_two_calls():
    from directaccesskernel_b200 import _lib

    stream = torch.cuda.current_stream().cuda_stream
    split, host = 64, 2
    for seed in (0, 1):  # two calls in a row; the second reuses the shared array
        q, kd, vd, kh, vh = _inputs(seed)
        B, H, S = q.shape[0], q.shape[1], kd.shape[2]
        ns = (S + split - 1) // split
        po = torch.empty(B, H, ns, 128, dtype=torch.float32, device="cuda")
        pml = torch.empty(B, H, ns, 2, dtype=torch.float32, device="cuda")
        ref_out = torch.empty(B, 1, H, 128, dtype=torch.float16, device="cuda")
        got_out = torch.full((B, 1, H, 128), float("nan"), dtype=torch.float16, device="cuda")
        a = _args(q, kd, vd, kh, vh, host, ref_out, split, po, pml)
        _lib.check(_lib.LIB.dak_attn_decode(ctypes.byref(a), stream), "dak_attn_decode")
        b = _args(q, kd, vd, kh, vh, host, got_out, split)
        _lib.check(_lib.LIB.dak_attn_decode_noalloc(ctypes.byref(b), stream), "dak_attn_decode_noalloc")
        torch.cuda.synchronize()
        got = got_out.float().cpu().numpy()
        assert not np.isnan(got).any()
        assert rel_err(got, ref_out.float().cpu().numpy()) < TOL
    assert _lib.device_status() == 0


def test_noalloc_rejects_calls_beyond_its_scratch():
    from directaccesskernel_b200 import _lib

    q, kd, vd, kh, vh = _inputs(2, B=2, Hq=4, Hkv=4, S=64, host=1)
    out = torch.empty(2, 1, 4, 128, dtype=torch.float16, device="cuda")
    a = _args(q, kd, vd, kh, vh, 1, out, 64)
    a.batch, a.num_q_heads, a.seq_len = 64, 64, 1 << 20  # 64 x 64 x 16384 splits x 130 floats
    st = _lib.LIB.dak_attn_decode_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.DAK_ERR_INVALID_ARG
    assert b"exceeds" in _lib.LIB.dak_last_error_message()
