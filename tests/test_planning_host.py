"""Host-side planning helpers (no GPU): the per-rank host fractions that balance
the host streams of a tensor-parallel decode, and the attention split size."""
import math

import pytest

import bench
from directaccesskernel_b200.attention import auto_split_size


def test_balanced_host_fractions_keep_the_mean_and_follow_bandwidth():
    bw = [35.0] * 4 + [23.0] * 4
    f = bench.balanced_host_fractions(0.81, bw)
    assert sum(f) / len(f) == pytest.approx(0.81)
    # host bytes / bandwidth equal on every rank: the host streams finish together
    t = [fi / b for fi, b in zip(f, bw)]
    assert max(t) == pytest.approx(min(t))


def test_balanced_host_fractions_clamp_and_redistribute():
    f = bench.balanced_host_fractions(0.9, [35.0] * 4 + [23.0] * 4)
    assert all(0.0 <= x <= 1.0 for x in f)
    assert f[:4] == [1.0] * 4
    assert sum(f) / len(f) == pytest.approx(0.9)
    g = bench.balanced_host_fractions(0.5, [100.0, 1.0], lo=0.3)
    assert g[1] == pytest.approx(0.3) and g[0] == pytest.approx(0.7)
    assert bench.balanced_host_fractions(0.4, [50.0, 50.0]) == pytest.approx([0.4, 0.4])


@pytest.mark.parametrize("batch,heads,seq", [(32, 1, 16394), (8, 8, 32768), (1, 8, 640), (3, 2, 75), (64, 8, 4096)])
def test_auto_split_size_fills_whole_waves(batch, heads, seq):
    sp = auto_split_size(batch, heads, seq, num_sms=148)
    assert sp % 64 == 0 and sp >= 64
    splits = math.ceil(seq / sp)
    ctas = batch * heads * splits
    # never worse than the old rule of about four waves
    want = max(1, (4 * 148 + batch * heads - 1) // (batch * heads))
    old = max(64, math.ceil(seq / want / 64) * 64)
    old_splits = math.ceil(seq / old)
    cost = lambda s, n: math.ceil(batch * heads * n / 148) * (s // 64 + 2)  # noqa: E731
    assert cost(sp, splits) <= cost(old, old_splits)
    assert ctas >= 1


def test_layer_roofline_terms():
    """The per-layer bound bench.py reports: HBM for the decode sweep (the tensor
    term is at most a quarter of it at M = 64), tensor cores for HBM-resident
    weights at prefill size, and the host link once half the rows are offloaded."""
    hbm, host, tf = 6452.5, 51.3, 1642.4
    for n, k in bench.LLAMA8B.values():
        for m in bench.TOKENS:
            which, t = bench.layer_roofline(m, n, k, 0, hbm, host, tf)
            assert which == "hbm"
            assert 2.0 * m * n * k / (tf * 1e12) <= 0.26 * t
        which, t = bench.layer_roofline(512, n, k, 0, hbm, host, tf)
        assert which == "tensor" and t == pytest.approx(2.0 * 512 * n * k / (tf * 1e12))
        half = n * k  # bytes: half of the 2 n k weight bytes
        which, t = bench.layer_roofline(512, n, k, half, hbm, host, tf)
        assert which == "host" and t == pytest.approx(half / (host * 1e9))


def test_rank_shape_matches_a_tp8_rank():
    """``bench.py --rank-of-tp 8`` builds one TP8 rank's layer shapes as a one-GPU
    model: its per-rank weight bytes equal a TP8 rank's (up to the replicated
    embedding, which holds one vocabulary shard instead of the full table)."""
    from directaccesskernel_b200 import decode
    from directaccesskernel_b200.llama_tp import LlamaShape

    full = LlamaShape.from_config(decode.llama_config("llama-3-70b"))
    r = bench.rank_shape(full, 8)
    assert (r.heads, r.kv_heads, r.ffn, r.hidden, r.head_dim) == (8, 1, 3584, 8192, 128)
    emb_full, emb_r = full.vocab * full.hidden * 2, r.vocab * r.hidden * 2
    assert r.weight_bytes_per_rank(1) - emb_r + emb_full == pytest.approx(full.weight_bytes_per_rank(8), rel=1e-3)
    assert r.kv_bytes_per_rank(1, 32, 16384) == full.kv_bytes_per_rank(8, 32, 16384)
    with pytest.raises(ValueError):
        bench.rank_shape(full, 3)


def _bench(args, env_extra=None, timeout=300):
    import json
    import os
    import subprocess
    import sys

    from conftest import REPO

    env = dict(os.environ, **(env_extra or {}))
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True, text=True,
                       timeout=timeout, env=env, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    return [json.loads(ln) for ln in lines]


def bench_config():
    import argparse

    import bench

    args = argparse.Namespace(workload="linear", tokens=None, ratios=None)
    return bench.linear_metric_config(*bench.linear_sweep(args), 1)[1]


def test_reference_arm_prints_one_contract_line():
    """`bench.py --impl reference` (the driver's reference arm): one JSON line on
    this arm's metric and unit, with the CPU baseline it timed and an e2e entry
    without host/device copies."""
    (line,) = _bench(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["metric"].startswith("offloaded GEMV effective weight GB/s")
    assert line["value"] > 0 and line["steps"] == 1
    cpu = line["cpu_baseline"]
    # The reference's own computation (torch F.linear on FP32 copies), with the
    # oracle port's figure beside it; the same config as the GPU arm's line.
    assert cpu["kind"] == "reference" and cpu["cores"] >= 1 and cpu["value"] == line["value"] and cpu["sample"]
    assert "F.linear" in cpu["sample"] and cpu["port_value"] > 0
    assert line["config"] == bench_config()
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    assert _bench(["--impl", "reference", "--steps", "1", "--warmup", "0"], {"RANK": "1", "WORLD_SIZE": "2"}) == []
