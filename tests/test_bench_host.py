"""Host-side pieces of bench.py's tensor-parallel linear sweep (no GPU): the
per-rank host fractions keep each layer's mean offload ratio, the parity check
flags a wrong output, and both arms describe the same workload."""
import argparse
import sys

import pytest
import torch

from conftest import REPO

sys.path.insert(0, str(REPO))
import bench  # noqa: E402


@pytest.mark.parametrize("ratio", [0.25, 0.5, 0.75])
@pytest.mark.parametrize("bws", [[55.0, 55.0], [35.0, 35.0, 35.0, 35.0, 23.0, 23.0, 23.0, 23.0], [50.0, 10.0]])
def test_host_fractions_keep_the_layer_ratio(ratio, bws):
    fr = bench.balanced_host_fractions(ratio, bws)
    assert sum(fr) / len(fr) == pytest.approx(ratio)
    assert all(0.0 <= f <= 1.0 for f in fr)
    # Unclamped ranks get host bytes in proportion to their bandwidth, so their
    # host streams end together.
    free = [f / b for f, b in zip(fr, bws) if 0.0 < f < 1.0]
    assert max(free) == pytest.approx(min(free))


def test_parity_flags_a_wrong_output():
    torch.manual_seed(0)
    w = (torch.randn(64, 32) * 0.02).half()
    x = torch.randn(4, 1, 32).half()
    layer = {"name": "t", "k": 32}
    ref = torch.nn.functional.linear(x.reshape(4, 32).float(), w.float())
    good = bench.linear_parity(torch, [layer], [(layer, 4)], [ref.half().reshape(4, 1, 64)], {"t": w},
                               {(4, 32): x})
    assert good["ok"] and good["max_rel_err"] < 1e-2
    bad = ref.clone()
    bad[2, 5] += 10 * ref.abs().max()
    res = bench.linear_parity(torch, [layer], [(layer, 4)], [bad.half().reshape(4, 1, 64)], {"t": w}, {(4, 32): x})
    assert not res["ok"]


@pytest.mark.parametrize("workload", ["linear", "prefill"])
@pytest.mark.parametrize("gpus", [1, 8])
def test_both_arms_describe_the_same_workload(workload, gpus):
    args = argparse.Namespace(workload=workload, tokens=None, ratios=None)
    prefill, tokens, ratios = bench.linear_sweep(args)
    metric, config = bench.linear_metric_config(prefill, tokens, ratios, gpus)
    assert config["layers_per_step"] == len(tokens) * len(ratios) * 4
    assert config["weight_bytes_per_step"] == len(tokens) * len(ratios) * 436207616
    assert ("tp8" in config["parallelism"]) == (gpus == 8)
    assert bench.linear_metric_config(prefill, tokens, ratios, gpus) == (metric, config)
