"""The fused decode-layer kernels (decode_ops) against transformers' Llama ops
computed by torch on the same 16-bit tensors."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ulps(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("with_residual", [False, True])
def test_rmsnorm(dtype, with_residual):
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    from directaccesskernel_b200.decode_ops import rmsnorm

    g = torch.Generator(device="cuda").manual_seed(0)
    rows, cols = 7, 8192
    x = torch.randn(rows, cols, generator=g, device="cuda").to(dtype)
    res = torch.randn(rows, cols, generator=g, device="cuda").to(dtype)
    w = (1 + 0.1 * torch.randn(cols, generator=g, device="cuda")).to(dtype)
    ref_mod = LlamaRMSNorm(cols, eps=1e-5).to("cuda", dtype)
    with torch.no_grad():
        ref_mod.weight.copy_(w)
        h = (x + res) if with_residual else x
        ref = ref_mod(h)
    if with_residual:
        state = res.clone()
        out = rmsnorm(x, w, 1e-5, residual=state)
        assert torch.equal(state, h)  # the fused add wrote x + residual back
    else:
        out = rmsnorm(x, w, 1e-5)
    assert _ulps(out, ref) < (2e-3 if dtype == torch.float16 else 1e-2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rope_qk_matches_transformers(dtype):
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    from directaccesskernel_b200.decode_ops import rope_qk

    B, hq, hkv, d, theta = 5, 8, 2, 128, 500000.0
    g = torch.Generator(device="cuda").manual_seed(1)
    qkv = torch.randn(B, (hq + 2 * hkv) * d, generator=g, device="cuda").to(dtype)
    pos = torch.tensor([0, 1, 17, 4095, 16390], dtype=torch.int32, device="cuda")
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).float().cuda() / d))
    q_out = torch.empty(B, hq, d, dtype=dtype, device="cuda")
    k_out = torch.empty(B, hkv, d, dtype=dtype, device="cuda")
    v_out = torch.empty(B, hkv, d, dtype=dtype, device="cuda")
    rope_qk(qkv, pos, inv_freq, hq, hkv, d, q_out, k_out, v_out)
    freqs = pos.float()[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(dtype)[:, None, None, :], emb.sin().to(dtype)[:, None, None, :]
    q = qkv[:, :hq * d].view(B, hq, 1, d)
    k = qkv[:, hq * d:(hq + hkv) * d].view(B, hkv, 1, d)
    rq, rk = apply_rotary_pos_emb(q, k, cos[:, 0], sin[:, 0], unsqueeze_dim=1)
    assert _ulps(q_out, rq[:, :, 0]) < 2e-3
    assert _ulps(k_out, rk[:, :, 0]) < 2e-3
    assert torch.equal(v_out.view(B, -1), qkv[:, (hq + hkv) * d:])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_silu_mul(dtype):
    from directaccesskernel_b200.decode_ops import silu_mul

    g = torch.Generator(device="cuda").manual_seed(2)
    gu = (3 * torch.randn(9, 2 * 3584, generator=g, device="cuda")).to(dtype)
    out = silu_mul(gu)
    ref = torch.nn.functional.silu(gu[:, :3584]) * gu[:, 3584:]
    assert _ulps(out, ref) < 2e-3
