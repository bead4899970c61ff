"""GPU parity of the split-tier linear kernels (CUDA-core and tcgen05 paths)
against the oracle, through the C ABI and through the reference-shaped API.

Tolerance (from the task's parity bar): normwise max relative error
max|y - y_ref| / max|y_ref| <= 1e-2 against FP32/FP64 accumulation; the
kernels accumulate in FP32 and round once to 16 bits, so the observed error is
about 1e-3."""

import numpy as np
import pytest
import torch

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _inputs(n_out, k, ntok, dtype=torch.float16, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    w = (torch.randn(n_out, k, generator=g) * 0.02).to(dtype)
    x = torch.randn(ntok, k, generator=g).to(dtype)
    return w, x


def _oracle(w, x):
    return oracle.linear(x.float().numpy(), w.float().numpy(), acc=np.float64)


def _split_run(w, x, host_cols, host_side="first", **kw):
    from directaccesskernel_b200 import runtime

    n_out, k = w.shape
    if host_side == "first":
        wh, wd = w[:host_cols], w[host_cols:]
        hoff, doff = 0, host_cols
    else:
        wh, wd = w[n_out - host_cols:], w[: n_out - host_cols]
        hoff, doff = n_out - host_cols, 0
    w_host = wh.t().contiguous().pin_memory() if host_cols > 0 else None
    w_dev = wd.t().contiguous().cuda() if host_cols < n_out else None
    xd = x.cuda()
    y = torch.full((x.shape[0], n_out), float("nan"), dtype=x.dtype, device="cuda")
    runtime.linear_split(xd, y, w_host, w_dev, hoff, doff, **kw)
    torch.cuda.synchronize()
    assert runtime.device_status() == 0
    return y.float().cpu().numpy()


@pytest.mark.parametrize("ntok", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("shape", [(256, 512), (320, 192), (4096, 1024), (1088, 4160)])
def test_cuda_core_path(shape, ntok):
    from directaccesskernel_b200 import _lib

    w, x = _inputs(*shape, ntok)
    ref = _oracle(w, x)
    for host_cols in (0, 64, shape[0] // 2 // 64 * 64, shape[0]):
        y = _split_run(w, x, host_cols, path=_lib.PATH_CUDA_CORE)
        assert not np.isnan(y).any()
        assert rel_err(y, ref) < TOL, (host_cols, rel_err(y, ref))


@pytest.mark.parametrize("ntok", [1, 9, 16, 17, 33, 64, 100, 128, 200, 256, 300])
@pytest.mark.parametrize("shape", [(256, 512), (384, 192), (4096, 1024), (1088, 4160)])
def test_tcgen05_path(shape, ntok):
    from directaccesskernel_b200 import _lib

    w, x = _inputs(*shape, ntok, seed=1)
    ref = _oracle(w, x)
    for host_cols in (0, 128, shape[0]):
        y = _split_run(w, x, host_cols, path=_lib.PATH_TCGEN05)
        assert not np.isnan(y).any()
        assert rel_err(y, ref) < TOL, (host_cols, rel_err(y, ref))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ntok", [257, 300, 512, 700, 1024])
@pytest.mark.parametrize("shape", [(256, 512), (384, 200), (1088, 4160)])
def test_wide_prefill_path(shape, ntok, dtype):
    """Batches of 257..512 tokens per chunk on a layer with host rows go to the
    wide kernel (each weight tile once for both 256-token halves); ragged
    batches, a K that is not a multiple of 64 and partial 64-feature boxes."""
    from directaccesskernel_b200 import _lib

    w, x = _inputs(*shape, ntok, dtype=dtype, seed=7)
    ref = _oracle(w, x)
    for host_cols in (64, 128, shape[0]):
        y = _split_run(w, x, host_cols, path=_lib.PATH_TCGEN05)
        assert not np.isnan(y).any()
        assert rel_err(y, ref) < TOL, (host_cols, rel_err(y, ref))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ntok", [1, 4, 16, 64])
def test_dtypes_and_host_side(dtype, ntok):
    w, x = _inputs(2048, 2048, ntok, dtype=dtype, seed=2)
    ref = _oracle(w, x)
    for side in ("first", "last"):
        y = _split_run(w, x, 1024, host_side=side)
        assert rel_err(y, ref) < TOL


@pytest.mark.parametrize("ntok", [1, 8, 32])
@pytest.mark.parametrize("sched", [
    dict(host_ctas=1, dev_ctas=1, host_ksplit=1, dev_ksplit=1),
    dict(host_ctas=3, dev_ctas=10, host_ksplit=1, dev_ksplit=2),
    dict(host_ctas=8, dev_ctas=64, host_ksplit=2, dev_ksplit=4),
    dict(host_ctas=16, dev_ctas=128, host_ksplit=4, dev_ksplit=8),
    dict(host_ctas=2, dev_ctas=7, host_ksplit=3, dev_ksplit=5),
])
def test_explicit_schedules(sched, ntok):
    w, x = _inputs(1536, 2048, ntok, seed=3)
    ref = _oracle(w, x)
    y = _split_run(w, x, 512, **sched)
    assert rel_err(y, ref) < TOL


def test_k_not_multiple_of_tile_and_tiny_k():
    for (n_out, k, ntok) in [(128, 8, 1), (128, 40, 3), (192, 72, 20), (64, 4104, 2)]:
        w, x = _inputs(n_out, k, ntok, seed=4)
        ref = _oracle(w, x)
        y = _split_run(w, x, 64)
        assert rel_err(y, ref) < TOL, (n_out, k, ntok)


def test_unaligned_strides_are_rejected():
    from directaccesskernel_b200 import runtime

    x = torch.randn(2, 100, dtype=torch.float16, device="cuda")[:, 1:]  # misaligned base
    y = torch.empty(2, 64, dtype=torch.float16, device="cuda")
    w = torch.randn(99, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="aligned|stride"):
        runtime.linear_split(x, y, None, w)


def test_pageable_host_weight_is_rejected():
    from directaccesskernel_b200 import runtime

    x = torch.randn(1, 64, dtype=torch.float16, device="cuda")
    y = torch.empty(1, 64, dtype=torch.float16, device="cuda")
    w = torch.randn(64, 64, dtype=torch.float16)  # not pinned
    with pytest.raises(RuntimeError, match="pinned"):
        runtime.linear_split(x, y, w, None)


# ------------------------------------------------------------ reference API
def _make_layer(cls, n_out, k, w):
    from directaccesskernel_b200.utils import get_smem_size

    lin = cls(k, n_out, smem_size=get_smem_size(), num_copy_blocks=128, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        lin.weight.copy_(w.cuda())
    return lin


@pytest.mark.parametrize("ntok", [1, 4, 8, 16, 64])
@pytest.mark.parametrize("cfg", [(0, 0, 16, 112, 1, 1), (64, 4032, 2, 128, 2, 2), (2048, 2048, 8, 64, 1, 4),
                                 (0, 0, 0, 0, 1, 1)])
def test_linear_horizontal_reference_api(cfg, ntok):
    from directaccesskernel_b200.layers import LinearHorizontal

    w, x = _inputs(4096, 4096, ntok, seed=5)
    ref = _oracle(w, x)
    lin = _make_layer(LinearHorizontal, 4096, 4096, w)
    h_m, d_m, hb, db, hs, ds = cfg
    lin.horizontal_split_weight(0.5, hb + db, hb, hs, ds, h_m, d_m)
    assert lin.weight_h.is_pinned() and lin.weight_d.is_cuda
    for _ in range(2):  # second call re-points the cached descriptors
        y = lin(x.cuda().view(ntok, 1, 4096))
        assert y.shape == (ntok, 1, 4096)
        assert rel_err(y.float().cpu().numpy().reshape(ntok, 4096), ref) < TOL


@pytest.mark.parametrize("device", ["cpu", "cuda"])
def test_single_tier_linear(device):
    from directaccesskernel_b200.layers import Linear

    w, x = _inputs(1024, 2048, 3, seed=6)
    ref = _oracle(w, x)
    lin = _make_layer(Linear, 1024, 2048, w)
    lin.move_weight_to_device(device)
    lin.config(64, 2)
    lin.build_tma_desc()
    y = lin(x.cuda())
    assert rel_err(y.float().cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("ntok", [300, 512, 700])
@pytest.mark.parametrize("blocks", [0, 64])
def test_single_tier_host_weight_prefill(ntok, blocks):
    """A whole weight in pinned host memory (linearLayer.py:72-80) at prefill
    batch sizes: the single-tier entry point serves it as the host tier, on the
    kernel that streams it once per 512 tokens; automatic and explicit plans."""
    from directaccesskernel_b200.layers import Linear, LinearMulticast

    w, x = _inputs(1024, 2048, ntok, seed=8)
    ref = _oracle(w, x)
    for cls in (Linear, LinearMulticast):
        lin = _make_layer(cls, 1024, 2048, w)
        lin.move_weight_to_device("cpu")
        if blocks and cls is Linear:
            lin.config(blocks, 2)
        lin.build_tma_desc()
        y = lin(x.cuda())
        assert rel_err(y.float().cpu().numpy(), ref) < TOL, cls.__name__


@pytest.mark.parametrize("prefill", [True, False])
@pytest.mark.parametrize("ntok", [5, 256, 512])
def test_multicast_layers(prefill, ntok):
    from directaccesskernel_b200.layers import LinearHorizontalMulticast, LinearMulticast

    w, x = _inputs(1024, 1024, ntok, seed=7)
    ref = _oracle(w, x)
    lin = _make_layer(LinearMulticast, 1024, 1024, w)
    lin.move_weight_to_device("cuda")
    lin.prefill = prefill
    assert rel_err(lin(x.cuda()).float().cpu().numpy(), ref) < TOL
    lin = _make_layer(LinearHorizontalMulticast, 1024, 1024, w)
    lin.horizontal_split_weight(0.25, 64, 8, 1, 1, 256, 768)
    lin.prefill = prefill
    assert rel_err(lin(x.cuda()).float().cpu().numpy(), ref) < TOL


def test_runtime_gemv_with_reference_helpers():
    """The call sequence of benchmark/benchmark_linear.py:199-226 (horizontal)."""
    from directaccesskernel_b200 import runtime
    from directaccesskernel_b200.config import TILE_K, TILE_M, TILE_N
    from directaccesskernel_b200.layers import LinearHorizontal
    from directaccesskernel_b200.utils import build_tma_wgmma_k, build_tma_wgmma_mn, get_smem_size, split_horizontal

    m, k, bsz = 4096, 4096, 8
    w, x = _inputs(m, k, bsz, seed=8)
    ref = _oracle(w, x)
    m_h, m_d = split_horizontal((m, k), 0.5)
    smem = runtime.set_smem_size(get_smem_size(), runtime.GEMV_HORIZONTAL)
    lin = LinearHorizontal(k, m, smem_size=smem, num_copy_blocks=32, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        lin.weight.copy_(w.cuda())
    lin.horizontal_split_weight(0.5, 32, 16, 1, 1, m_h, m_d)
    lin.build_tma_desc()
    inp = x.cuda().view(bsz, 1, k)
    _, dx = build_tma_wgmma_k(inp.view(-1, k), TILE_K, TILE_N)
    out = torch.zeros(bsz, 1, m, device="cuda", dtype=torch.float16)
    _, dy = build_tma_wgmma_mn(out.view(-1, m), TILE_M, TILE_N)
    runtime.gemv_horizontal(lin.w_desc_h, lin.w_desc_d, dx, dy, m_h, m_d, bsz, k, 32, 16, smem, 1, 1)
    torch.cuda.synchronize()
    assert rel_err(out.float().cpu().numpy().reshape(bsz, m), ref) < TOL
    # The reference's MAPE check (benchmark_linear.py:264-266), against fp16 nn.Linear.
    ref16 = torch.nn.functional.linear(inp, w.cuda())
    mape = (torch.abs(out - ref16) / (torch.abs(ref16) + 1e-6)).float().mean() * 100
    assert mape.item() < 1.0


def test_cuda_graph_capture_and_replay():
    from directaccesskernel_b200.layers import LinearHorizontal

    w, x = _inputs(2048, 2048, 1, seed=9)
    ref = _oracle(w, x)
    lin = _make_layer(LinearHorizontal, 2048, 2048, w)
    lin.horizontal_split_weight(0.25, 0, 0, 1, 1)
    xin = x.cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        lin(xin)  # warm up: builds descriptors and tile maps
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = lin(xin)
    for seed in (10, 11):
        _, x2 = _inputs(2048, 2048, 1, seed=seed)
        xin.copy_(x2.cuda())
        g.replay()
        torch.cuda.synchronize()
        assert rel_err(y.float().cpu().numpy(), _oracle(w, x2)) < TOL


def test_config1_full_size_last_rows_on_host():
    """W [4096, 4096] ~ N(0, 0.02), x [1, 4096] ~ N(0, 1),
    last 2048 rows in pinned host memory, seed 0."""
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(4096, 4096, generator=g) * 0.02).half()
    x = torch.randn(1, 4096, generator=g).half()
    ref = _oracle(w, x)
    y = _split_run(w, x, 2048, host_side="last")
    assert rel_err(y, ref) < TOL


LLAMA8B = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}


@pytest.mark.parametrize("name", list(LLAMA8B))
def test_config2_llama8b_sweep(name):
    """BASELINE config 2 at full size: every M and offload ratio."""
    from directaccesskernel_b200.utils import split_horizontal

    n, k = LLAMA8B[name]
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(n, k, generator=g) * 0.02).half()
    xs = torch.randn(64, k, generator=g).half()
    wf = w.float().numpy()
    for m in (1, 4, 16, 64):
        x = xs[:m]
        ref = (x.float().numpy() @ wf.T)
        for r in (0.0, 0.25, 0.5, 0.75, 1.0):
            h_m, _ = split_horizontal((n, k), r)
            y = _split_run(w, x, h_m)
            assert rel_err(y, ref) < TOL, (name, m, r, rel_err(y, ref))


@pytest.mark.parametrize("ntok", [65, 128, 200, 256, 300, 512, 700, 1024])
@pytest.mark.parametrize("name", list(LLAMA8B))
def test_token_sliced_hbm_only_prefill(name, ntok):
    """HBM-only layers above 64 tokens run as grid rows of 64 to 256 tokens,
    up to 512 tokens per launch (ragged last row and ragged last launch
    included); every row writes only its own tokens."""
    n, k = LLAMA8B[name]
    g = torch.Generator().manual_seed(ntok)
    w = (torch.randn(n, k, generator=g) * 0.02).half()
    x = torch.randn(ntok, k, generator=g).half()
    ref = (x.float() @ w.float().t()).numpy()
    y = _split_run(w, x, 0)
    assert not np.isnan(y).any()
    assert rel_err(y, ref) < TOL, (name, ntok, rel_err(y, ref))


@pytest.mark.parametrize("ntok", [256, 250])
@pytest.mark.parametrize("n_out,k", [(28864, 1024), (38464, 512), (4096 + 64, 1024)])
def test_hbm_only_multi_tile_ctas(n_out, k, ntok):
    """256-token HBM-only launches whose CTAs hold two or three tiles, the last
    of one 64-feature box, and a narrow layer that gets token rows."""
    w, x = _inputs(n_out, k, ntok, seed=n_out + ntok)
    ref = _oracle(w, x)
    y = _split_run(w, x, 0)
    assert not np.isnan(y).any()
    assert rel_err(y, ref) < TOL, rel_err(y, ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ntok", [257, 300, 512])
@pytest.mark.parametrize("n_out,k", [(28672, 1024), (28864, 1024), (38464, 512), (20480 + 192, 640)])
def test_paired_wide_hbm_only(n_out, k, ntok, dtype):
    """HBM-only layers wide enough to fill the SMs take 257..512 tokens on the
    wide kernel's paired mode: each CTA applies one 256-token row to two
    128-feature tiles.  Box counts that leave a last unit of one to three
    64-feature boxes, and a ragged last token row, included."""
    w, x = _inputs(n_out, k, ntok, dtype=dtype, seed=n_out + ntok)
    ref = _oracle(w, x)
    y = _split_run(w, x, 0)
    assert not np.isnan(y).any()
    assert rel_err(y, ref) < TOL, rel_err(y, ref)


def test_token_slices_are_planned(tmp_path):
    """The plan trace shows the narrow HBM-only layer of 4096 features cut into
    four 64-token rows at 256 tokens and into four 128-token rows of one launch
    at 512 tokens, no rows when it has host rows, and a wide HBM-only layer
    (224 tiles) left whole at 256 tokens and paired at 512."""
    import os
    import subprocess
    import sys

    from conftest import REPO

    code = (
        "import torch\n"
        "from directaccesskernel_b200 import runtime\n"
        "x = torch.randn(256, 1024, device='cuda').half()\n"
        "w = (torch.randn(1024, 4096) * 0.02).half()\n"
        "y = torch.empty(256, 4096, device='cuda').half()\n"
        "runtime.linear_split(x, y, None, w.cuda())\n"
        "runtime.linear_split(x, y, w[:, :512].contiguous().pin_memory(), w[:, 512:].contiguous().cuda(), 0, 512)\n"
        "wide = (torch.randn(1024, 28672, device='cuda') * 0.02).half()\n"
        "runtime.linear_split(x, torch.empty(256, 28672, device='cuda').half(), None, wide)\n"
        "x2 = torch.randn(512, 1024, device='cuda').half()\n"
        "runtime.linear_split(x2, torch.empty(512, 4096, device='cuda').half(), None, w.cuda())\n"
        "runtime.linear_split(x2, torch.empty(512, 28672, device='cuda').half(), None, wide)\n"
        "torch.cuda.synchronize()\n"
        "assert runtime.device_status() == 0\n")
    env = dict(os.environ, DAK_B200_TRACE_PLAN="1", PYTHONPATH=str(REPO))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr
    plans = [line for line in r.stderr.splitlines() if line.startswith("[dak plan] tcgen05 ntok=256")]
    assert len(plans) == 3, r.stderr
    assert "x 4 rows of 64 tokens |" in plans[0], plans[0]
    assert "x 1 rows of 256 tokens |" in plans[1], plans[1]
    assert "x 1 rows of 256 tokens |" in plans[2], plans[2]
    # 512 tokens of the narrow layer: one launch of four 128-token rows.
    wide_plans = [line for line in r.stderr.splitlines() if line.startswith("[dak plan] tcgen05 ntok=512")]
    assert len(wide_plans) == 1 and "x 4 rows of 128 tokens |" in wide_plans[0], r.stderr
    # 512 tokens of the wide layer (224 tiles): the paired mode, 56 CTAs x 2 rows.
    paired = [line for line in r.stderr.splitlines() if line.startswith("[dak plan] wide paired ntok=512")]
    assert len(paired) == 1 and "dev ctas=56 x 2 rows" in paired[0], r.stderr


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ntok", [1, 4, 32, 64, 100, 256])
@pytest.mark.parametrize("f,k", [(3584, 8192), (512, 1024), (48, 200)])
def test_gated_linear(f, k, ntok, dtype):
    """linear_split(glu=True) on interleaved gate/up rows: silu(x g^T) * (x u^T)
    against the oracle, with every row in HBM, the first rows on the host, and
    every row on the host."""
    from directaccesskernel_b200 import runtime

    g = torch.Generator().manual_seed(f + ntok)
    gate = (torch.randn(f, k, generator=g) * 0.02).to(dtype)
    up = (torch.randn(f, k, generator=g) * 0.02).to(dtype)
    x = torch.randn(ntok, k, generator=g).to(dtype)
    xg = oracle.linear(x.float().numpy(), gate.float().numpy(), acc=np.float64)
    xu = oracle.linear(x.float().numpy(), up.float().numpy(), acc=np.float64)
    ref = xg / (1.0 + np.exp(-xg)) * xu
    wt = runtime.interleave_gate_up(gate, up).t().contiguous()  # [K, 2F]
    for host_cols in (0, 64 if 2 * f > 64 else 0, 2 * f):
        wh = wt[:, :host_cols].contiguous().pin_memory() if host_cols else None
        wd = wt[:, host_cols:].contiguous().cuda() if host_cols < 2 * f else None
        y = torch.full((ntok, f), float("nan"), dtype=dtype, device="cuda")
        runtime.linear_split(x.cuda(), y, wh, wd, 0, host_cols, glu=True)
        torch.cuda.synchronize()
        assert runtime.device_status() == 0
        got = y.float().cpu().numpy()
        assert not np.isnan(got).any()
        assert rel_err(got, ref) < TOL, (host_cols, rel_err(got, ref))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_token_slices_and_gated_linear_in_a_cuda_graph(dtype):
    """Token-sliced launches (down-like: 4 rows of 64 tokens) and the gated
    linear, captured once in a CUDA graph and replayed on new activations."""
    from directaccesskernel_b200 import runtime

    g = torch.Generator().manual_seed(21)
    w = (torch.randn(4096, 1024, generator=g) * 0.02).to(dtype)
    gate = (torch.randn(512, 1024, generator=g) * 0.02).to(dtype)
    up = (torch.randn(512, 1024, generator=g) * 0.02).to(dtype)
    wt = w.t().contiguous().cuda()
    gt = runtime.interleave_gate_up(gate, up).t().contiguous().cuda()
    xin = torch.zeros(256, 1024, dtype=dtype, device="cuda")
    y = torch.empty(256, 4096, dtype=dtype, device="cuda")
    act = torch.empty(256, 512, dtype=dtype, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        runtime.linear_split(xin, y, None, wt)
        runtime.linear_split(xin, act, None, gt, glu=True)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        runtime.linear_split(xin, y, None, wt)
        runtime.linear_split(xin, act, None, gt, glu=True)
    for seed in (22, 23):
        x = torch.randn(256, 1024, generator=torch.Generator().manual_seed(seed)).to(dtype)
        xin.copy_(x.cuda())
        graph.replay()
        torch.cuda.synchronize()
        assert runtime.device_status() == 0
        assert rel_err(y.float().cpu().numpy(), _oracle(w, x)) < TOL
        xg, xu = _oracle(gate, x), _oracle(up, x)
        assert rel_err(act.float().cpu().numpy(), xg / (1.0 + np.exp(-xg)) * xu) < TOL
