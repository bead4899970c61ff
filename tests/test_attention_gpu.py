"""GPU parity of the split-KV decode attention (batch-split `_C.decode` form and
paged form) against the oracle and the reference's recorded outputs.

Tolerance (from the task's parity bar): normwise max relative error
max|o - o_ref| / max|o_ref| <= 2e-3 against softmax attention in FP32."""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import gen, golden_npz, rel_err

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _pinned(a: np.ndarray, dtype=torch.float16) -> torch.Tensor:
    return torch.from_numpy(a).to(dtype).pin_memory()


@pytest.mark.parametrize("name", ["mha_split", "mha_mask", "all_host", "all_gpu", "mha_fp16"])
def test_decode_matches_reference_hook_outputs(name):
    from directaccesskernel_b200.attention import decode

    d = golden_npz("attention_ref.npz")
    B, H, S, host, fp16, use_mask = (int(v) for v in d[f"{name}_cfg"])
    seeds = [int(s) for s in d[f"{name}_seeds"]]
    q = gen(seeds[0], (B, H, 1, 128)) / np.float16(math.sqrt(128))
    k = gen(seeds[1], (B, H, S, 128))
    v = gen(seeds[2], (B, H, S, 128))
    mask = torch.from_numpy(d[f"{name}_mask"]).cuda() if use_mask else None
    out = decode(torch.from_numpy(q).cuda(), torch.from_numpy(k[host:]).cuda(), torch.from_numpy(v[host:]).cuda(),
                 _pinned(k[:host]), _pinned(v[:host]), host, mask, 1.0 / math.sqrt(128), 64)
    torch.cuda.synchronize()
    ref = d[f"{name}_out"]
    # The fp16 case's reference rounds P to fp16 before P.V (the hook's eager path).
    assert rel_err(out.float().cpu().numpy(), ref) < (4e-3 if fp16 else TOL)


@pytest.mark.parametrize("B,Hq,Hkv,S,host,split", [
    (1, 1, 1, 1, 0, 64), (2, 4, 4, 63, 1, 64), (2, 4, 4, 65, 1, 64), (3, 8, 2, 1000, 2, 256),
    (4, 32, 8, 4097, 2, 512), (2, 16, 2, 300, 0, 128), (2, 8, 8, 128, 2, 64), (8, 64, 8, 2048, 4, 1024),
])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_random(B, Hq, Hkv, S, host, split, dtype):
    from directaccesskernel_b200.attention import decode

    rng = np.random.default_rng(B * 1000 + S)
    q = (rng.standard_normal((B, Hq, 1, 128)) / math.sqrt(128)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, S, 128)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, S, 128)).astype(np.float32)
    qt = torch.from_numpy(q).to(dtype)
    kt = torch.from_numpy(k).to(dtype)
    vt = torch.from_numpy(v).to(dtype)
    out = decode(qt.cuda(), kt[host:].cuda(), vt[host:].cuda(), kt[:host].pin_memory(), vt[:host].pin_memory(),
                 host, None, 1.0 / math.sqrt(128), split)
    ref = oracle.decode_attention(qt.float().numpy(), kt.float().numpy(), vt.float().numpy(), None,
                                  1.0 / math.sqrt(128))
    assert rel_err(out.float().cpu().numpy(), ref) < (8e-3 if dtype == torch.bfloat16 else TOL)


def test_decode_with_mask_and_strided_cache():
    """A StaticCache slice: batch/head strides larger than the packed ones, additive mask."""
    from directaccesskernel_b200.attention import decode

    rng = np.random.default_rng(5)
    B, H, S, Smax = 4, 4, 192, 256
    big_k = torch.from_numpy(rng.standard_normal((B, H, Smax, 128)).astype(np.float16))
    big_v = torch.from_numpy(rng.standard_normal((B, H, Smax, 128)).astype(np.float16))
    q = torch.from_numpy((rng.standard_normal((B, H, 1, 128)) / 11.3).astype(np.float16))
    mask = np.zeros((B, 1, 1, S), np.float32)
    mask[1, ..., 100:] = -1e30
    mask[3, ..., :50] = -1e30
    kd, vd = big_k[2:, :, :S].cuda(), big_v[2:, :, :S].cuda()
    kh, vh = big_k[:2, :, :S].pin_memory(), big_v[:2, :, :S].pin_memory()
    out = decode(q.cuda(), kd, vd, kh, vh, 2, torch.from_numpy(mask).cuda(), 0.1, 64)
    ref = oracle.decode_attention(q.float().numpy(), big_k[:, :, :S].float().numpy(), big_v[:, :, :S].float().numpy(),
                                  mask, 0.1)
    assert rel_err(out.float().cpu().numpy(), ref) < TOL


def test_decode_argument_errors():
    from directaccesskernel_b200.attention import decode

    q = torch.zeros(2, 2, 1, 128, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, 2, 64, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="host_size"):
        decode(q, k, k, None, None, 3)
    with pytest.raises(RuntimeError, match="key_host is required"):
        decode(q, k, k, None, None, 1)
    with pytest.raises(RuntimeError, match="pinned"):
        kh = torch.zeros(1, 2, 64, 128, dtype=torch.float16)
        decode(q, k, k, kh, kh, 1)
    with pytest.raises(RuntimeError, match="head_dim"):
        decode(torch.zeros(2, 2, 1, 64, dtype=torch.float16, device="cuda"), k, k, None, None, 1)
    with pytest.raises(RuntimeError, match="multiple of 64"):
        decode(q, torch.zeros(2, 2, 64, 128, dtype=torch.float16, device="cuda"),
               torch.zeros(2, 2, 64, 128, dtype=torch.float16, device="cuda"), split_size=100)


def _paged_setup(B, Hq, Hkv, seq_lens, P, host_frac, seed, dtype=torch.float16):
    rng = np.random.default_rng(seed)
    max_pages = max((s + P - 1) // P for s in seq_lens)
    q = (rng.standard_normal((B, Hq, 128)) / math.sqrt(128)).astype(np.float32)
    npg = sum((s + P - 1) // P for s in seq_lens)
    kpool = rng.standard_normal((npg, Hkv, P, 128)).astype(np.float32)
    vpool = rng.standard_normal((npg, Hkv, P, 128)).astype(np.float32)
    on_host = rng.random(npg) < host_frac
    perm = rng.permutation(npg)  # pages of a sequence are scattered over the pools
    dev_idx = {p: i for i, p in enumerate([p for p in perm if not on_host[p]])}
    host_idx = {p: i for i, p in enumerate([p for p in perm if on_host[p]])}
    kd = np.zeros((max(1, len(dev_idx)), Hkv, P, 128), np.float32)
    vd = np.zeros_like(kd)
    kh = np.zeros((max(1, len(host_idx)), Hkv, P, 128), np.float32)
    vh = np.zeros_like(kh)
    table = np.full((B, max_pages), 0x7FFFFFFF, np.int32)  # entries past a sequence are never read
    g = 0
    for b, s in enumerate(seq_lens):
        for j in range((s + P - 1) // P):
            if on_host[g]:
                kh[host_idx[g]], vh[host_idx[g]] = kpool[g], vpool[g]
                table[b, j] = -1 - host_idx[g]
            else:
                kd[dev_idx[g]], vd[dev_idx[g]] = kpool[g], vpool[g]
                table[b, j] = dev_idx[g]
            g += 1
    cast = lambda a: torch.from_numpy(a).to(dtype)  # noqa: E731
    return dict(q=cast(q), kd=cast(kd), vd=cast(vd), kh=cast(kh), vh=cast(vh), table=table,
                seq=np.array(seq_lens, np.int32))


@pytest.mark.parametrize("B,Hq,Hkv,seq_lens,P,host_frac,split", [
    (1, 4, 1, [16], 16, 0.5, 64),
    (2, 8, 2, [1, 333], 16, 0.5, 64),
    (3, 32, 8, [700, 64, 1025], 16, 0.5, 256),
    (2, 8, 8, [500, 500], 32, 1.0, 128),
    (2, 8, 4, [640, 100], 64, 0.0, 128),
    (4, 16, 2, [2048, 1, 999, 1500], 16, 0.3, None),
])
def test_paged_decode_mixed_tiers(B, Hq, Hkv, seq_lens, P, host_frac, split):
    from directaccesskernel_b200.attention import decode_paged

    s = _paged_setup(B, Hq, Hkv, seq_lens, P, host_frac, seed=B * 7 + P)
    has_dev = (s["table"][s["table"] != 0x7FFFFFFF] >= 0).any()
    has_host = (s["table"] < 0).any()
    out = decode_paged(s["q"].cuda(), s["kd"].cuda() if has_dev else None, s["vd"].cuda() if has_dev else None,
                       s["kh"].pin_memory() if has_host else None, s["vh"].pin_memory() if has_host else None,
                       torch.from_numpy(s["table"]).cuda(), torch.from_numpy(s["seq"]).cuda(), 1.0 / math.sqrt(128),
                       split)
    ref = oracle.paged_decode(s["q"].float().numpy(), s["kd"].float().numpy(), s["vd"].float().numpy(),
                              s["kh"].float().numpy(), s["vh"].float().numpy(), s["table"], s["seq"],
                              1.0 / math.sqrt(128))
    assert rel_err(out.float().cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,Hq,Hkv,seq_lens,P,host_frac,split", [
    (2, 8, 2, [1, 333], 16, 0.5, 64),
    (3, 32, 8, [700, 64, 1025], 16, 0.5, 256),
    (4, 16, 2, [2048, 1, 999, 1500], 64, 0.3, 192),
])
def test_paged_decode_with_in_kernel_merge(B, Hq, Hkv, seq_lens, P, host_frac, split, dtype):
    """With merge counters the last split of each (sequence, KV head) merges in
    the attention kernel: the output is bitwise the separate merge kernel's,
    over several calls in a row and CUDA-graph replays, and the counters are
    left at zero."""
    from directaccesskernel_b200 import runtime
    from directaccesskernel_b200.attention import decode_paged

    s = _paged_setup(B, Hq, Hkv, seq_lens, P, host_frac, seed=B * 11 + P, dtype=dtype)
    has_dev = (s["table"][s["table"] != 0x7FFFFFFF] >= 0).any()
    has_host = (s["table"] < 0).any()
    args = (s["q"].cuda(), s["kd"].cuda() if has_dev else None, s["vd"].cuda() if has_dev else None,
            s["kh"].pin_memory() if has_host else None, s["vh"].pin_memory() if has_host else None,
            torch.from_numpy(s["table"]).cuda(), torch.from_numpy(s["seq"]).cuda(), 1.0 / math.sqrt(128), split)
    ref = decode_paged(*args)
    counters = torch.zeros(B * Hkv, dtype=torch.int32, device="cuda")
    out = torch.full_like(ref, float("nan"))
    for _ in range(3):
        decode_paged(*args, out=out, merge_counters=counters)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert int(counters.abs().sum()) == 0
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side), torch.cuda.graph(graph):
        decode_paged(*args, out=out, merge_counters=counters)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert int(counters.abs().sum()) == 0
    assert runtime.device_status() == 0


def test_in_kernel_merge_rejects_bad_counters():
    from directaccesskernel_b200.attention import decode_paged

    s = _paged_setup(2, 8, 2, [300, 300], 16, 0.0, seed=5)
    args = (s["q"].cuda(), s["kd"].cuda(), s["vd"].cuda(), None, None, torch.from_numpy(s["table"]).cuda(),
            torch.from_numpy(s["seq"]).cuda(), 1.0 / math.sqrt(128), 64)
    with pytest.raises(RuntimeError, match="merge_counters"):
        decode_paged(*args, merge_counters=torch.zeros(4, dtype=torch.int64, device="cuda"))
    with pytest.raises(RuntimeError, match="merge_counters"):
        decode_paged(*args, merge_counters=torch.zeros(3, dtype=torch.int32, device="cuda"))
    with pytest.raises(RuntimeError, match="merge_counters"):
        decode_paged(*args, merge_counters=torch.zeros(4, dtype=torch.int32).pin_memory())


def test_hf_hook_decode_through_registry():
    import opt_attention
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    opt_attention.register()
    fn = ALL_ATTENTION_FUNCTIONS["vdcores_opt"]
    rng = np.random.default_rng(3)
    B, H, S = 4, 4, 256
    q = torch.from_numpy((rng.standard_normal((B, H, 1, 128)) / 11.3).astype(np.float16))
    k = torch.from_numpy(rng.standard_normal((B, H, S, 128)).astype(np.float16))
    v = torch.from_numpy(rng.standard_normal((B, H, S, 128)).astype(np.float16))
    module = torch.nn.Module().eval()
    out, w = fn(module, q.cuda(), k[2:].cuda(), v[2:].cuda(), None, dropout=0.0, scaling=0.125,
                key_host=k[:2].pin_memory(), value_host=v[:2].pin_memory(), host_size=2)
    assert w is None and out.shape == (B, 1, H, 128)
    ref = oracle.decode_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), None, 0.125)
    assert rel_err(out.float().cpu().numpy(), ref) < TOL


def test_config3_full_size_subset():
    """batch 8, 32/8 heads, head_dim 128, context 32768,
    16-token pages with half of them in pinned host memory.  All rows are
    computed; rows 0 and 5 are checked against the oracle."""
    from directaccesskernel_b200.attention import decode_paged

    B, Hq, Hkv, S, P = 8, 32, 8, 32768, 16
    g = torch.Generator(device="cuda").manual_seed(0)
    npg = B * S // P
    kpool = torch.randn(npg, Hkv, P, 128, generator=g, device="cuda", dtype=torch.float16)
    vpool = torch.randn(npg, Hkv, P, 128, generator=g, device="cuda", dtype=torch.float16)
    q = torch.randn(B, Hq, 128, generator=g, device="cuda", dtype=torch.float16)
    perm = torch.randperm(npg, generator=torch.Generator().manual_seed(0))
    host_pages = perm[: npg // 2].sort().values
    dev_pages = perm[npg // 2:].sort().values
    kh = kpool[host_pages.cuda()].cpu().pin_memory()
    vh = vpool[host_pages.cuda()].cpu().pin_memory()
    kd = kpool[dev_pages.cuda()].contiguous()
    vd = vpool[dev_pages.cuda()].contiguous()
    table = torch.empty(npg, dtype=torch.int32)
    table[host_pages] = -1 - torch.arange(len(host_pages), dtype=torch.int32)
    table[dev_pages] = torch.arange(len(dev_pages), dtype=torch.int32)
    table = table.view(B, S // P)
    seq = torch.full((B,), S, dtype=torch.int32)
    out = decode_paged(q, kd, vd, kh, vh, table.cuda(), seq.cuda(), 1.0 / math.sqrt(128))
    torch.cuda.synchronize()
    for b in (0, 5):
        k = kpool.view(B, S // P, Hkv, P, 128)[b].permute(1, 0, 2, 3).reshape(Hkv, S, 128)
        v = vpool.view(B, S // P, Hkv, P, 128)[b].permute(1, 0, 2, 3).reshape(Hkv, S, 128)
        ref = oracle.decode_attention(q[b][None, :, None].float().cpu().numpy(), k[None].float().cpu().numpy(),
                                      v[None].float().cpu().numpy(), None, 1.0 / math.sqrt(128))
        assert rel_err(out[b].float().cpu().numpy(), ref[0, 0]) < TOL
