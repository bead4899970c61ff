"""End-to-end decode over stock transformers causal LMs with offloaded linears.

The same plumbing as the reference's decode benchmarks (benchmark/benchmark_opt.py:
137-460, benchmark/benchmark_llama.py): a transformers model whose decoder
linears are replaced by the offloaded modules (``linear_replacement``), placed
between pinned host memory and HBM (``placement.place_model``), prefilled with a
prompt, then decoded greedily with a ``StaticCache`` and one CUDA graph per step.

What differs from the reference harness:
  * weights are random (N(0, std) linears and embeddings, unit norms) and are
    created on the meta device first, so a 131 GB model is never materialised
    on the host; each tensor is allocated and filled on the GPU;
  * placement can take an HBM budget (``hbm_budget_bytes``) instead of a ratio;
  * the decode loop reports per-step latency from CUDA events, as the reference
    does (benchmark_opt.py:361-418): TBT, tokens/s = batch / TBT, and effective
    weight bandwidth = model bytes / TBT.
"""
from __future__ import annotations

import dataclasses
import time

import torch
from torch import nn

from .linear_replacement import LinearReplacementConfig, replace_llama_linears, replace_opt_linears
from .placement import ModelPlacementStats, place_model


# ------------------------------------------------------------------ configs
def opt_config(name: str = "opt-66b", **overrides):
    """OPT architectures of the reference's OPT benchmarks (facebook/opt-*)."""
    from transformers import OPTConfig

    shapes = {
        "opt-66b": dict(hidden_size=9216, num_hidden_layers=64, ffn_dim=36864, num_attention_heads=72),
        "opt-30b": dict(hidden_size=7168, num_hidden_layers=48, ffn_dim=28672, num_attention_heads=56),
        "opt-6.7b": dict(hidden_size=4096, num_hidden_layers=32, ffn_dim=16384, num_attention_heads=32),
    }
    kw = dict(shapes[name], vocab_size=50272, max_position_embeddings=2048, do_layer_norm_before=True,
              enable_bias=True, word_embed_proj_dim=shapes[name]["hidden_size"], init_std=0.02)
    kw.update(overrides)
    return OPTConfig(**kw)


def llama_config(name: str = "llama-3-70b", **overrides):
    """Llama-3 architectures of the reference's Llama benchmarks."""
    from transformers import LlamaConfig

    shapes = {
        "llama-3-70b": dict(hidden_size=8192, num_hidden_layers=80, num_attention_heads=64,
                            num_key_value_heads=8, intermediate_size=28672),
        "llama-3-8b": dict(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
                           num_key_value_heads=8, intermediate_size=14336),
    }
    kw = dict(shapes[name], vocab_size=128256, max_position_embeddings=131072, rope_theta=500000.0,
              rms_norm_eps=1e-5, initializer_range=0.02, tie_word_embeddings=False)
    kw.update(overrides)
    return LlamaConfig(**kw)


# ------------------------------------------------------------ construction
def _is_norm(mod: nn.Module) -> bool:
    return isinstance(mod, nn.LayerNorm) or "RMSNorm" in type(mod).__name__


@torch.no_grad()
def materialize_random_(model: nn.Module, *, device="cuda", std: float = 0.02, seed: int = 0) -> nn.Module:
    """Allocate every meta parameter on ``device`` and fill it: norms get weight 1 and
    bias 0, biases 0, everything else N(0, std).  Shared (tied) parameters stay shared.
    Rotary-embedding modules are rebuilt on the device from the model config.

    Parameters are visited in module order, so two models with the same module tree
    (the offloaded one and its unreplaced "vanila" twin) get identical weights from
    the same seed."""
    gen = torch.Generator(device=device).manual_seed(seed)
    memo: dict[int, nn.Parameter] = {}
    for mod in model.modules():
        for name, p in list(mod.named_parameters(recurse=False)):
            if p is None or p.device.type != "meta":
                continue
            new = memo.get(id(p))
            if new is None:
                t = torch.empty(p.shape, dtype=p.dtype, device=device)
                if _is_norm(mod):
                    t.fill_(1.0 if name == "weight" else 0.0)
                elif name == "bias":
                    t.zero_()
                else:
                    t.normal_(0.0, std, generator=gen)
                new = nn.Parameter(t, requires_grad=False)
                memo[id(p)] = new
            setattr(mod, name, new)
    for parent in list(model.modules()):
        for cname, child in list(parent.named_children()):
            if "RotaryEmbedding" in type(child).__name__ and any(b.device.type == "meta" for b in child.buffers()):
                setattr(parent, cname, type(child)(config=model.config, device=device))
    for mod in model.modules():
        for name, b in list(mod.named_buffers(recurse=False)):
            if b is not None and b.device.type == "meta":
                raise RuntimeError(f"buffer {name} of {type(mod).__name__} was left on the meta device")
    return model


def _family(config) -> str:
    mt = getattr(config, "model_type", "")
    if mt == "opt":
        return "opt"
    if mt == "llama":
        return "llama"
    raise ValueError(f"unsupported model_type {mt!r} (opt or llama)")


def build_offloaded_model(config, *, linear_type: str = "horizontal", offload_ratio: float | None = None,
                          hbm_budget_bytes: int | None = None, dtype=torch.float16, std: float = 0.02,
                          seed: int = 0, device="cuda", host_side: str = "first",
                          attn_implementation: str = "sdpa") -> tuple[nn.Module, ModelPlacementStats]:
    """A random-init transformers causal LM whose decoder linears are offloaded.

    ``linear_type`` is a reference linear type ("horizontal", "host", "multicast",
    "horizontal_multicast"), or "vanila" for the unreplaced model (all linears
    nn.Linear in HBM, the reference's offload_ratio == 0 path).  Placement uses
    ``offload_ratio`` or ``hbm_budget_bytes`` (the host fraction of the replaced
    linears that makes everything fit the budget)."""
    from transformers import AutoModelForCausalLM

    config._attn_implementation = attn_implementation
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(config, dtype=dtype)
    family = _family(config)
    if linear_type != "vanila":
        repl = LinearReplacementConfig(linear_type, device="meta", dtype=dtype, drop_bias=False)
        (replace_opt_linears if family == "opt" else replace_llama_linears)(model, repl)
    materialize_random_(model, device=device, std=std, seed=seed)
    model.eval()
    if linear_type == "vanila":
        n = sum(p.numel() * p.element_size() for p in model.parameters())
        return model, ModelPlacementStats(0, n, 0.0)
    if hbm_budget_bytes is not None:
        stats = place_model(model, None, hbm_budget_bytes=hbm_budget_bytes, device=device, host_side=host_side)
    else:
        stats = place_model(model, offload_ratio, device=device, host_side=host_side)
    torch.cuda.synchronize()
    return model, stats


# ------------------------------------------------------------------ decode
@dataclasses.dataclass
class DecodeResult:
    tokens: torch.Tensor          # [B, prompt + generated]
    step_ms: list[float]          # per timed decode step (CUDA events)
    prefill_ms: float
    logits: list[torch.Tensor]    # per decode step [B, V] (when keep_logits)

    @property
    def tbt_ms(self) -> float:
        return sum(self.step_ms) / max(1, len(self.step_ms))

    def tokens_per_s(self, batch: int) -> float:
        return batch * 1e3 / self.tbt_ms if self.step_ms else 0.0


class GreedyDecoder:
    """Prefill + greedy decode with a StaticCache and one CUDA graph per step, the
    loop of benchmark_opt.py:244-360 (fixed-shape token, mask and position buffers
    updated in place between replays)."""

    def __init__(self, model: nn.Module, batch: int, max_cache_len: int, *, graph: bool = True,
                 dtype=torch.float16, device="cuda"):
        from transformers.cache_utils import StaticCache

        self.model = model
        self.B = batch
        self.max_len = max_cache_len
        self.graph_enabled = graph
        self.device = device
        self.cache = StaticCache(config=model.config, max_cache_len=max_cache_len)
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=device)
        self.mask = torch.zeros(batch, max_cache_len, dtype=torch.long, device=device)
        self.pos = torch.zeros(batch, 1, dtype=torch.long, device=device)
        self.cache_pos = torch.zeros(1, dtype=torch.long, device=device)
        self.graph = None
        self.out = None
        self.cur = 0

    def _cache_counters(self) -> list[torch.Tensor]:
        """The device tensors that hold each cache layer's write position
        (transformers' StaticLayer.cumulative_length)."""
        out = []
        for layer in getattr(self.cache, "layers", []):
            c = getattr(layer, "cumulative_length", None)
            if isinstance(c, torch.Tensor):
                out.append(c)
        return out

    def _step_forward(self):
        return self.model(input_ids=self.ids, attention_mask=self.mask, position_ids=self.pos, use_cache=True,
                          past_key_values=self.cache, cache_position=self.cache_pos, logits_to_keep=1)

    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor) -> torch.Tensor:
        B, L = input_ids.shape
        if B != self.B or L >= self.max_len:
            raise ValueError(f"prompt [{B}, {L}] does not fit batch {self.B} / cache {self.max_len}")
        self.cache.reset()
        self.mask.zero_()
        self.mask[:, :L] = 1
        out = self.model(input_ids=input_ids, attention_mask=self.mask[:, :L], use_cache=True,
                         past_key_values=self.cache, cache_position=torch.arange(L, device=self.device),
                         logits_to_keep=1)
        logits = out.logits[:, -1, :]
        nxt = torch.argmax(logits, dim=-1)
        self.ids[:, 0] = nxt
        self.mask[:, L] = 1
        self.pos[:, 0] = L
        self.cache_pos[0] = L
        self.cur = L
        return logits

    @torch.inference_mode()
    def step(self) -> torch.Tensor:
        """One decode step on the current buffers; returns the step's logits [B, V]."""
        if self.graph_enabled:
            if self.graph is None:
                # The static cache advances its write position with a device counter
                # on every forward; the warm-up forwards must not move it.
                saved = [c.clone() for c in self._cache_counters()]
                for _ in range(2):  # lazy init and allocator warm-up before capture
                    self._step_forward()
                torch.cuda.synchronize()
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph):
                    self.out = self._step_forward()
                for c, v in zip(self._cache_counters(), saved):
                    c.copy_(v)
            self.graph.replay()
            return self.out.logits[:, -1, :]
        return self._step_forward().logits[:, -1, :]

    @torch.inference_mode()
    def advance(self, logits: torch.Tensor, forced: torch.Tensor | None = None) -> torch.Tensor:
        """Choose the next token (greedy, or ``forced``) and move the buffers on."""
        nxt = torch.argmax(logits, dim=-1) if forced is None else forced.to(self.ids.device)
        self.cur += 1
        if self.cur >= self.max_len:
            raise RuntimeError("static cache is full")
        self.ids[:, 0] = nxt
        self.mask[:, self.cur] = 1
        self.pos[:, 0] += 1
        self.cache_pos[0] = self.cur
        return nxt

    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, new_tokens: int, *, keep_logits: bool = False,
                 forced: torch.Tensor | None = None, warmup_steps: int = 0) -> DecodeResult:
        """Prefill, then ``new_tokens`` decode steps; the first ``warmup_steps`` decode
        steps are not timed.  ``forced`` [B, new_tokens] teacher-forces the tokens fed
        (column 0 right after prefill), for logit comparisons between two models."""
        t0 = time.perf_counter()
        logits = self.prefill(input_ids)
        torch.cuda.synchronize()
        prefill_ms = (time.perf_counter() - t0) * 1e3
        toks = [input_ids]
        first = torch.argmax(logits, dim=-1) if forced is None else forced[:, 0].to(input_ids.device)
        self.ids[:, 0] = first
        toks.append(first[:, None])
        kept, times = [], []
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(new_tokens)]
        for i in range(new_tokens):
            ev[i][0].record()
            lg = self.step()
            ev[i][1].record()
            if keep_logits:
                kept.append(lg.float().clone())
            if i + 1 < new_tokens:
                nxt = self.advance(lg, None if forced is None else forced[:, i + 1])
                toks.append(nxt[:, None])
            else:
                toks.append(torch.argmax(lg, dim=-1)[:, None])
        torch.cuda.synchronize()
        times = [ev[i][0].elapsed_time(ev[i][1]) for i in range(warmup_steps, new_tokens)]
        return DecodeResult(torch.cat(toks, 1), times, prefill_ms, kept)


def model_weight_bytes(model: nn.Module) -> int:
    return sum(p.numel() * p.element_size() for p in model.parameters())


def decode_roofline_ms(stats: ModelPlacementStats, hbm_gbs: float, host_gbs: float) -> float:
    """Lower bound of one decode step: every weight byte is read once, the host bytes
    over the host link and the rest from HBM, concurrently (KV and activations are
    negligible at the reference's decode configs with batch 1)."""
    return max(stats.device_bytes / (hbm_gbs * 1e9), stats.host_bytes / (host_gbs * 1e9)) * 1e3


def random_prompt(batch: int, length: int, vocab: int, seed: int = 0, device="cuda") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (batch, length), generator=g).to(device)


__all__ = [
    "opt_config", "llama_config", "materialize_random_", "build_offloaded_model",
    "GreedyDecoder", "DecodeResult", "model_weight_bytes", "decode_roofline_ms", "random_prompt",
]
