"""The writer side of the tiered paged KV cache (dak_kv_append_paged) on the GPU:
appends land in the right device or pinned host page, a cache built token by
token decodes like the dense oracle, and bad table entries are recorded in the
device error word instead of being written."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu


def _pools(pages_dev, pages_host, hkv, P, D=128, dtype=torch.float16, seed=0):
    g = torch.Generator().manual_seed(seed)
    kd = torch.randn(pages_dev, hkv, P, D, generator=g).to(dtype).cuda()
    vd = torch.randn(pages_dev, hkv, P, D, generator=g).to(dtype).cuda()
    kh = torch.randn(pages_host, hkv, P, D, generator=g).to(dtype).pin_memory()
    vh = torch.randn(pages_host, hkv, P, D, generator=g).to(dtype).pin_memory()
    return kd, vd, kh, vh


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_append_lands_in_the_named_page(dtype):
    from directaccesskernel_b200.attention import kv_append_paged

    B, Hkv, P, D = 4, 2, 16, 128
    kd, vd, kh, vh = _pools(5, 5, Hkv, P, D, dtype)
    table = torch.tensor([[0, -1, 3], [-2, 1, -5], [4, -3, 2], [-4, -5, 0]], dtype=torch.int32)
    pos = torch.tensor([20, 2, 40, 10], dtype=torch.int32)  # host, host, device, host
    g = torch.Generator().manual_seed(1)
    kn = torch.randn(B, Hkv, D, generator=g).to(dtype)
    vn = torch.randn(B, Hkv, D, generator=g).to(dtype)
    exp = [t.cpu().clone() for t in (kd, vd, kh, vh)]
    for b in range(B):
        e = int(table[b, pos[b] // P])
        slot = int(pos[b]) % P
        if e >= 0:
            exp[0][e, :, slot] = kn[b]
            exp[1][e, :, slot] = vn[b]
        else:
            exp[2][-1 - e, :, slot] = kn[b]
            exp[3][-1 - e, :, slot] = vn[b]
    kv_append_paged(kn.cuda(), vn.cuda(), kd, vd, kh, vh, table.cuda(), pos.cuda())
    torch.cuda.synchronize()
    for got, want in zip((kd, vd, kh, vh), exp):
        assert torch.equal(got.cpu(), want)


def test_cache_built_token_by_token_decodes_like_the_oracle():
    from directaccesskernel_b200 import runtime
    from directaccesskernel_b200.attention import decode_paged, kv_append_paged

    B, Hq, Hkv, P, D, L = 3, 8, 2, 16, 128, 75
    npg = (L + P - 1) // P
    kd, vd, kh, vh = _pools(B * npg, B * npg, Hkv, P, D)
    # Alternate tiers page by page, differently per sequence.
    table = torch.empty(B, npg, dtype=torch.int32)
    for b in range(B):
        for j in range(npg):
            table[b, j] = (b * npg + j) if (b + j) % 2 else -1 - (b * npg + j)
    tab = table.cuda()
    g = torch.Generator().manual_seed(3)
    K = torch.randn(B, Hkv, L, D, generator=g).half()
    V = torch.randn(B, Hkv, L, D, generator=g).half()
    for t in range(L):
        pos = torch.full((B,), t, dtype=torch.int32, device="cuda")
        kv_append_paged(K[:, :, t].contiguous().cuda(), V[:, :, t].contiguous().cuda(), kd, vd, kh, vh, tab, pos)
    q = torch.randn(B, Hq, D, generator=g).half()
    seq = torch.full((B,), L, dtype=torch.int32, device="cuda")
    out = decode_paged(q.cuda(), kd, vd, kh, vh, tab, seq, 1 / math.sqrt(D), 64)
    ref = oracle.decode_attention(q.numpy()[:, :, None, :], K.numpy(), V.numpy(), None, 1 / math.sqrt(D))[:, 0]
    assert rel_err(out.float().cpu().numpy(), ref) < 2e-3
    assert runtime.device_status() == 0


def test_bad_entries_are_recorded_not_written():
    from directaccesskernel_b200 import _lib, runtime
    from directaccesskernel_b200.attention import kv_append_paged

    Hkv, P = 2, 16
    kd, vd, kh, vh = _pools(2, 2, Hkv, P)
    before = [t.cpu().clone() for t in (kd, vd, kh, vh)]
    table = torch.tensor([[0, 7], [-9, 1]], dtype=torch.int32, device="cuda")  # device page 7, host page 8 do not exist
    pos = torch.tensor([20, 5], dtype=torch.int32, device="cuda")
    kn = torch.randn(2, Hkv, 128).half().cuda()
    assert runtime.device_status() == 0
    kv_append_paged(kn, kn.clone(), kd, vd, kh, vh, table, pos)
    assert runtime.device_status(clear=True) == _lib.DAK_ERR_INVALID_ARG
    for got, want in zip((kd, vd, kh, vh), before):
        assert torch.equal(got.cpu(), want)
    # A position past the table is caught too.
    kv_append_paged(kn, kn.clone(), kd, vd, kh, vh, table, torch.tensor([40, 0], dtype=torch.int32, device="cuda"))
    assert runtime.device_status(clear=True) == _lib.DAK_ERR_INVALID_ARG


def test_append_argument_errors():
    from directaccesskernel_b200.attention import kv_append_paged

    kd, vd, kh, vh = _pools(2, 2, 2, 16)
    table = torch.zeros(1, 2, dtype=torch.int32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    kn = torch.randn(1, 2, 128).half().cuda()
    with pytest.raises(RuntimeError):
        kv_append_paged(kn, kn, kd, vd, kh.clone(), vh, table, pos)  # unpinned host pool
    with pytest.raises(RuntimeError):
        kv_append_paged(kn.float(), kn.float(), kd, vd, kh, vh, table, pos)
    with pytest.raises(RuntimeError):
        kv_append_paged(kn, kn, kd, None, kh, vh, table, pos)


def test_writer_matches_the_reference_pinned_static_cache():
    """Fed the update sequence that tests/golden/kv_cache.npz ran through the
    reference's PinnedStaticCache (app/python/pinned_static_cache.py:47-107), one
    token per sequence and call, the paged writer holds exactly the reference
    cache's tokens, in host and device pages, for both layers."""
    from conftest import KV_WRITTEN, gen, golden_npz, kv_cache_updates, kv_page_table

    from directaccesskernel_b200 import runtime
    from directaccesskernel_b200.attention import kv_append_paged

    d = golden_npz("kv_cache.npz")
    layers, B, hidden, heads, hkv, S = (int(v) for v in d["cfg"])
    D, P = hidden // heads, 8
    npg = S // P
    table = kv_page_table(B, npg)
    tab = torch.from_numpy(table.astype(np.int32)).cuda()
    pools = [_pools(B * npg, B * npg, hkv, P, D, seed=20 + layer) for layer in range(layers)]
    for pos, seed in kv_cache_updates():
        k = gen(seed, (B, hkv, len(pos), D))
        v = gen(seed + 1000, (B, hkv, len(pos), D))
        for layer in range(layers):
            kd, vd, kh, vh = pools[layer]
            for t, p in enumerate(pos):
                kv_append_paged(torch.from_numpy(np.ascontiguousarray(k[:, :, t])).cuda(),
                                torch.from_numpy(np.ascontiguousarray(v[:, :, t])).cuda(), kd, vd, kh, vh, tab,
                                torch.full((B,), p, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    assert runtime.device_status() == 0
    for layer in range(layers):
        kd, vd, kh, vh = (t.cpu().numpy() for t in pools[layer])
        for b in range(B):
            kb = oracle.paged_gather(kd, kh, table[b], S)
            vb = oracle.paged_gather(vd, vh, table[b], S)
            assert np.array_equal(kb[:, KV_WRITTEN], d[f"k{layer}"][b][:, KV_WRITTEN])
            assert np.array_equal(vb[:, KV_WRITTEN], d[f"v{layer}"][b][:, KV_WRITTEN])


@pytest.mark.parametrize("host_pool", [True, False])
def test_paged_attention_bounds_table_entries(host_pool):
    """A block-table entry past its pool, or naming a tier without a pool, reads
    zeros and sets DAK_ERR_INVALID_ARG in the error word; the other pages are
    read as usual."""
    from directaccesskernel_b200 import _lib, runtime
    from directaccesskernel_b200.attention import decode_paged

    B, Hq, Hkv, P, D, npg = 2, 8, 2, 16, 128, 6
    kd, vd, kh, vh = _pools(npg, npg, Hkv, P, D, seed=9)
    if not host_pool:
        kh = vh = None
    table = np.array([[0, 1, npg, 2, 3, 4], [5, -1, -1 - npg, 0, 1, 2]], dtype=np.int32)
    if not host_pool:
        table[1] = [5, -1, 3, 0, 1, 2]  # -1 names a host page, and there is no host pool
    bad = {(0, 2), (1, 1)} if not host_pool else {(0, 2), (1, 2)}
    g = torch.Generator().manual_seed(4)
    q = (torch.randn(B, Hq, D, generator=g) / math.sqrt(D)).half()
    S = npg * P
    runtime.device_status(True)
    out = decode_paged(q.cuda(), kd, vd, kh, vh, torch.from_numpy(table).cuda(),
                       torch.full((B,), S, dtype=torch.int32, device="cuda"), 1 / math.sqrt(D), 64)
    assert runtime.device_status(True) == _lib.DAK_ERR_INVALID_ARG
    kdn, vdn = kd.cpu().numpy(), vd.cpu().numpy()
    khn = kh.numpy() if kh is not None else None
    vhn = vh.numpy() if vh is not None else None
    K = np.zeros((B, Hkv, S, D), np.float16)
    V = np.zeros((B, Hkv, S, D), np.float16)
    for b in range(B):
        for j in range(npg):
            if (b, j) in bad:
                continue  # reads zeros
            e = int(table[b, j])
            K[b, :, j * P:(j + 1) * P] = kdn[e] if e >= 0 else khn[-1 - e]
            V[b, :, j * P:(j + 1) * P] = vdn[e] if e >= 0 else vhn[-1 - e]
    ref = oracle.decode_attention(q.numpy()[:, :, None, :], K, V, None, 1 / math.sqrt(D))[:, 0]
    assert rel_err(out.float().cpu().numpy(), ref) < 2e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_rope_append_matches_rope_then_append(dtype):
    """dak_rope_kv_append writes q_out and every pool byte exactly as dak_rope_qk
    followed by dak_kv_append_paged do, with pages in both tiers; a bad table
    entry is recorded in the error word and nothing is written for it."""
    from directaccesskernel_b200 import _lib, runtime
    from directaccesskernel_b200.attention import kv_append_paged, rope_kv_append
    from directaccesskernel_b200.decode_ops import rope_qk

    B, Hq, Hkv, P, D = 5, 8, 2, 16, 128
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, generator=g, device="cuda").to(dtype)
    inv_freq = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.int64).float().cuda() / D))
    table = torch.tensor([[0, -1, 3], [-2, 1, -5], [4, -3, 2], [-4, -5, 0], [1, 2, -1]], dtype=torch.int32,
                         device="cuda")
    pos = torch.tensor([20, 2, 40, 10, 33], dtype=torch.int32, device="cuda")
    ref = _pools(5, 5, Hkv, P, D, dtype, seed=3)
    got = [t.clone() if t.is_cuda else t.clone().pin_memory() for t in ref]
    q_ref = torch.empty(B, Hq, D, dtype=dtype, device="cuda")
    k_new = torch.empty(B, Hkv, D, dtype=dtype, device="cuda")
    v_new = torch.empty_like(k_new)
    rope_qk(qkv, pos, inv_freq, Hq, Hkv, D, q_ref, k_new, v_new)
    kv_append_paged(k_new, v_new, *ref, table, pos)
    q_got = torch.empty_like(q_ref)
    rope_kv_append(qkv, pos, inv_freq, Hq, Hkv, D, q_got, *got, table)
    torch.cuda.synchronize()
    assert runtime.device_status() == 0
    assert torch.equal(q_got, q_ref)
    for a, b in zip(got, ref):
        assert torch.equal(a.cpu(), b.cpu())
    # An entry past its pool is recorded and skipped; both paths leave the
    # same bytes (sequence 1's token would land on host page 8 of 5).
    bad = table.clone()
    bad[1, 0] = -9
    k_new2, v_new2 = torch.empty_like(k_new), torch.empty_like(v_new)
    rope_qk(qkv, pos + 1, inv_freq, Hq, Hkv, D, q_ref, k_new2, v_new2)
    kv_append_paged(k_new2, v_new2, *ref, bad, pos + 1)
    assert runtime.device_status(clear=True) == _lib.DAK_ERR_INVALID_ARG
    rope_kv_append(qkv, pos + 1, inv_freq, Hq, Hkv, D, q_got, *got, bad)
    assert runtime.device_status(clear=True) == _lib.DAK_ERR_INVALID_ARG
    assert torch.equal(q_got, q_ref)
    for a, b in zip(got, ref):
        assert torch.equal(a.cpu(), b.cpu())
