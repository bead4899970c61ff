"""Host-side checks of the end-to-end decode harness (no GPU): model sizes and
HBM-budget placement arithmetic at BASELINE configs 4 and 5 on the meta device,
and the seeded materialisation that makes the offloaded model and its vanila
twin identical."""
from __future__ import annotations

import torch
from transformers import AutoModelForCausalLM

from directaccesskernel_b200 import decode
from directaccesskernel_b200.linear_replacement import (LinearReplacementConfig, replace_llama_linears,
                                                        replace_opt_linears)
from directaccesskernel_b200.placement import offload_ratio_for_budget


def _meta(cfg, replace=None):
    with torch.device("meta"):
        m = AutoModelForCausalLM.from_config(cfg, dtype=torch.float16)
    if replace is not None:
        replace(m, LinearReplacementConfig("horizontal", device="meta", dtype=torch.float16, drop_bias=False))
    return m


def test_opt66b_budget_split():
    """Config 4: OPT-66B (~131.4 GB fp16) under a 96 GB HBM budget puts ~35.4 GB
    of linear weights (r ~ 0.27) on the host."""
    m = _meta(decode.opt_config("opt-66b"), replace_opt_linears)
    total = sum(p.numel() for p in m.parameters()) * 2
    assert abs(total / 1e9 - 131.44) < 0.05
    r = offload_ratio_for_budget(m, 96 * 10**9)
    lin = sum(mod.weight.numel() * 2 for mod in m.modules() if hasattr(mod, "horizontal_split_weight"))
    assert abs(r - 0.2717) < 1e-3
    assert abs(r * lin / 1e9 - 35.44) < 0.05


def test_llama70b_sizes():
    """Config 5: Llama-3-70B architecture, ~70.55 B parameters."""
    m = _meta(decode.llama_config("llama-3-70b"))
    n = sum(p.numel() for p in m.parameters())
    assert abs(n / 1e9 - 70.55) < 0.01
    assert m.config.num_key_value_heads == 8 and m.config.head_dim == 128


def test_seeded_twins_are_identical():
    for cfg, repl in ((decode.opt_config("opt-6.7b", hidden_size=128, num_hidden_layers=2, ffn_dim=256,
                                         num_attention_heads=4, word_embed_proj_dim=128, vocab_size=300),
                       replace_opt_linears),
                      (decode.llama_config("llama-3-8b", hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                                           num_key_value_heads=2, intermediate_size=256, vocab_size=300),
                       replace_llama_linears)):
        a = decode.materialize_random_(_meta(cfg), device="cpu", seed=4)
        b = decode.materialize_random_(_meta(cfg, repl), device="cpu", seed=4)
        pa, pb = dict(a.named_parameters()), dict(b.named_parameters())
        assert pa.keys() == pb.keys()
        assert all(torch.equal(pa[k], pb[k]) for k in pa)
        assert all(p.device.type == "cpu" for p in b.parameters())
        assert all(bf.device.type == "cpu" for bf in b.buffers())
