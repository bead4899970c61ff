"""Host-side arithmetic of the tensor-parallel Llama decoder (no GPU): per-rank
bytes at BASELINE config 5, the HBM-budget host fraction, and the weight and
vocabulary sharding checked against the unsharded layer."""
import pytest
import torch

from directaccesskernel_b200 import decode
from directaccesskernel_b200.llama_tp import LlamaShape, TPLlamaDecoder, budget_fraction, vocab_rows_per_rank


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


def _cpu_rank(shape, rank, world):
    """A TPLlamaDecoder rank reduced to its sharding state, on the CPU in float64
    (no kernels: the linears are kept as plain weight matrices)."""
    dec = object.__new__(TPLlamaDecoder)
    torch.nn.Module.__init__(dec)
    dec.s, dec.rank, dec.world = shape, rank, world
    dec.hq, dec.hkv, dec.ffn_r = shape.heads // world, shape.kv_heads // world, shape.ffn // world
    dec.vocab_r = vocab_rows_per_rank(shape.vocab, world)
    dec.device, dec.dtype = "cpu", torch.float64
    dec._make_linear = lambda w: w
    return dec



@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_layer_shards_compose_to_the_full_layer(world):
    """Column-parallel q/k/v and gate/up, row-parallel o and down: the ranks'
    outputs concatenated (column) or summed (row) equal the unsharded layer, and
    every query head of a rank reads a KV head of the same rank."""
    s = LlamaShape(hidden=64, layers=1, heads=16, kv_heads=8, head_dim=8, ffn=96, vocab=300,
                   rope_theta=1e4, eps=1e-5)
    g = torch.Generator().manual_seed(0)
    rnd = lambda *shape: torch.randn(*shape, generator=g, dtype=torch.float64)  # noqa: E731
    d = s.head_dim
    full = {"q": rnd(s.heads * d, s.hidden), "k": rnd(s.kv_heads * d, s.hidden), "v": rnd(s.kv_heads * d, s.hidden),
            "o": rnd(s.hidden, s.heads * d), "gate": rnd(s.ffn, s.hidden), "up": rnd(s.ffn, s.hidden),
            "down": rnd(s.hidden, s.ffn)}
    x = rnd(3, s.hidden)
    attn = rnd(3, s.heads * d)  # stands in for the attention output
    silu = torch.nn.functional.silu
    q_parts, k_parts, v_parts, o_sum, mlp_sum = [], [], [], 0, 0
    for r in range(world):
        dec = _cpu_rank(s, r, world)
        sh = dec._shard_layer(full, 0)
        qkv = x @ sh["qkv"].T
        qd, kd = dec.hq * d, dec.hkv * d
        q_parts.append(qkv[:, :qd])
        k_parts.append(qkv[:, qd:qd + kd])
        v_parts.append(qkv[:, qd + kd:])
        o_sum = o_sum + attn[:, r * qd:(r + 1) * qd] @ sh["o"].T
        g, u = dec.split_gate_up(x @ sh["gate_up"].T)
        mlp_sum = mlp_sum + (silu(g) * u) @ sh["down"].T
        group = s.heads // s.kv_heads
        for i in range(dec.hq):
            assert (r * dec.hq + i) // group // dec.hkv == r
    torch.testing.assert_close(torch.cat(q_parts, 1), x @ full["q"].T)
    torch.testing.assert_close(torch.cat(k_parts, 1), x @ full["k"].T)
    torch.testing.assert_close(torch.cat(v_parts, 1), x @ full["v"].T)
    torch.testing.assert_close(o_sum, attn @ full["o"].T)
    torch.testing.assert_close(mlp_sum, (silu(x @ full["gate"].T) * (x @ full["up"].T)) @ full["down"].T)


@pytest.mark.parametrize("vocab", [300, 3000, 50272, 128256])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_vocab_shards_tile_the_vocabulary(world, vocab):
    """lm_head shards: whole 64-row tiles, zero padding only on the last ranks,
    and the ranks' valid rows cover the vocabulary exactly once in order."""
    s = LlamaShape(hidden=16, layers=1, heads=8, kv_heads=8, head_dim=2, ffn=16, vocab=vocab,
                   rope_theta=1e4, eps=1e-5)
    head = torch.arange(vocab, dtype=torch.float64)[:, None].expand(vocab, s.hidden).contiguous() + 1
    covered = []
    for r in range(world):
        dec = _cpu_rank(s, r, world)
        dec._set_head(torch.zeros(vocab, s.hidden), torch.ones(s.hidden), head)
        assert dec.vocab_r % 64 == 0 and dec.lm_head.shape == (dec.vocab_r, s.hidden)
        rows = dec.lm_head[:dec.vocab_valid, 0] - 1
        covered.extend(int(v) for v in rows)
        assert torch.all(dec.lm_head[dec.vocab_valid:] == 0)
    assert covered == list(range(vocab))


def test_kernel_launch_count_per_step():
    s = LlamaShape.from_config(decode.llama_config("llama-3-70b"))
    dec = _cpu_rank(s, 0, 8)
    dec.layers = list(range(20))
    dec.max_ctx, dec.split = 16384 + 64, 1024
    # Per layer: 4 linears (gate_up applies the SiLU gate: 3584 FFN features a
    # rank), rotary with the KV append, attention (which merges its own
    # splits) and 2 RMSNorms.
    assert dec.fuse_glu
    assert dec.kernel_launches_per_step() == 1 + 20 * 8 + 1
    dec.split = dec.max_ctx  # one split: the same launches
    assert dec.kernel_launches_per_step() == 1 + 20 * 8 + 1
    dec.fuse_glu = False  # an FFN width that is not whole 16-feature blocks: a SiLU-gate kernel too
    assert dec.kernel_launches_per_step() == 1 + 20 * 9 + 1
