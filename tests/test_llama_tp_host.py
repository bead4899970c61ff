"""Host-side arithmetic of the tensor-parallel Llama decoder (no GPU): per-rank
bytes at BASELINE config 5 and the HBM-budget host fraction."""
from directaccesskernel_b200 import decode
from directaccesskernel_b200.llama_tp import LlamaShape, budget_fraction


def test_config5_bytes_per_rank():
    s = LlamaShape.from_config(decode.llama_config("llama-3-70b"))
    assert (s.head_dim, s.kv_heads, s.ffn) == (128, 8, 28672)
    # 141.1 GB of fp16 weights in total; the embedding and the norms are
    # replicated on every rank, everything else is split 8 ways.
    w1 = s.weight_bytes_per_rank(1)
    assert abs(w1 / 1e9 - 141.1) < 0.2
    replicated = s.vocab * s.hidden * 2 + (2 * s.layers + 1) * s.hidden * 2
    assert (s.weight_bytes_per_rank(8) - replicated) * 8 + replicated == w1
    # KV at batch 32 x 16384 tokens: 327,680 B per token -> 171.8 GB.
    assert abs(s.kv_bytes_per_rank(1, 32, 16384) / 1e9 - 171.8) < 0.1
    assert s.kv_bytes_per_rank(8, 32, 16384) * 8 == s.kv_bytes_per_rank(1, 32, 16384)


def test_config5_budget_fractions():
    s = LlamaShape.from_config(decode.llama_config("llama-3-70b"))
    f = {g: budget_fraction(s, g, 32, 16384, 60 * 10**9) for g in (1, 2, 4, 8)}
    assert f[8] == 0.0                      # 39 GB per GPU fits the budget
    assert 0.2 < f[4] < 0.26                # ~18 GB per GPU on the host
    assert 0.6 < f[2] < 0.63
    assert 0.8 < f[1] < 0.82
