"""Tensor-parallel Llama decode with offloaded weights and a tiered paged KV cache.

BASELINE config 5 (Llama-3-70B architecture, batch 32, context 16384, a per-GPU
HBM budget that forces both weights and KV partly onto the host) on one box of
B200s.  Each rank holds 1/G of every layer Megatron-style:
  * q/k/v (merged) and gate/up (merged) are column-parallel: the rank owns
    Hq/G query heads, Hkv/G KV heads and FFN/G intermediate features;
  * o and down are row-parallel; their partial products are summed with one
    NCCL all-reduce each (the only inter-GPU traffic besides the greedy pick);
  * lm_head is column-parallel over the vocabulary; the greedy token is the
    maximum of the ranks' (value, index) pairs.
Every linear is an offloaded module (``layers.LinearHorizontal``): its host rows
sit in pinned memory and stream over this GPU's own host link.  The KV cache is
paged (64-token pages): the first pages of every sequence live in pinned host
memory, the rest in HBM; ``attention.rope_kv_append`` rotates each new token's
k and writes it with v straight into its page, and ``attention.decode_paged``
reads both tiers in one launch.  A decode step, greedy pick included, is one CUDA graph.

The layer arithmetic follows transformers' Llama (RMSNorm in FP32, rotary
embedding in the activation dtype, SiLU-gated MLP), which is also what the
reference's vanila_llama.py runs (app/python/llama/vanila_llama.py:227-400);
the element-wise steps are the fused kernels of ``decode_ops``.
"""
from __future__ import annotations

import contextlib
import dataclasses
import math

import torch
import torch.distributed as dist
from torch import nn

from .attention import auto_split_size, decode_paged, rope_kv_append

# Tokens per KV page.  One page of one KV head is a TMA box of page x 64 dims per
# half head; 64-token pages give 8 KB boxes, which stream from HBM about twice
# as fast as the 2 KB boxes of 16-token pages.
PAGE = 64


@dataclasses.dataclass
class LlamaShape:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float
    eps: float

    @classmethod
    def from_config(cls, cfg) -> "LlamaShape":
        hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        rope = getattr(cfg, "rope_parameters", None) or getattr(cfg, "rope_scaling", None) or {}
        theta = rope.get("rope_theta", getattr(cfg, "rope_theta", None))
        if theta is None:
            theta = 10000.0
        if rope.get("rope_type", "default") != "default":
            raise ValueError(f"rope_type {rope.get('rope_type')!r} is not supported (default rotary only)")
        return cls(cfg.hidden_size, cfg.num_hidden_layers, cfg.num_attention_heads, cfg.num_key_value_heads, hd,
                   cfg.intermediate_size, cfg.vocab_size, float(theta), float(cfg.rms_norm_eps))

    def weight_bytes_per_rank(self, world: int, dtype_bytes: int = 2) -> int:
        """Bytes of this rank's linears, norms and the replicated embedding."""
        h, d = self.hidden, self.head_dim
        per_layer = (h * (self.heads + 2 * self.kv_heads) * d + self.heads * d * h + 3 * h * self.ffn) // world
        vocab_r = -(-self.vocab // world)
        return dtype_bytes * (self.layers * (per_layer + 2 * h) + h + self.vocab * h + vocab_r * h)

    def kv_bytes_per_rank(self, world: int, batch: int, ctx: int, dtype_bytes: int = 2) -> int:
        pages = -(-ctx // PAGE)
        return dtype_bytes * 2 * self.layers * batch * pages * PAGE * (self.kv_heads // world) * self.head_dim


def vocab_rows_per_rank(vocab: int, world: int) -> int:
    """lm_head rows each rank holds: the vocabulary split G ways, rounded up to
    whole 64-row tiles.  Rows past the vocabulary are zero and never take part in
    the greedy pick."""
    return -(-vocab // (world * 64)) * 64


def budget_fraction(shape: LlamaShape, world: int, batch: int, ctx: int, hbm_budget_bytes: int) -> float:
    """Host fraction f of both weights and KV such that (1 - f) x (this rank's weights
    + KV) fits the per-GPU HBM budget (0 when everything fits)."""
    total = shape.weight_bytes_per_rank(world) + shape.kv_bytes_per_rank(world, batch, ctx)
    return max(0.0, 1.0 - hbm_budget_bytes / total)


class _Layer(nn.Module):
    def __init__(self, qkv, o, gate_up, down, in_w, post_w):
        super().__init__()
        self.qkv, self.o, self.gate_up, self.down = qkv, o, gate_up, down
        self.in_w = nn.Parameter(in_w, requires_grad=False)
        self.post_w = nn.Parameter(post_w, requires_grad=False)


class TPLlamaDecoder(nn.Module):
    """One rank of a tensor-parallel Llama decoder (see the module docstring).

    ``weight_offload`` is the host fraction of every linear shard (split by
    ``LinearHorizontal`` at 64-feature granularity); ``kv_host_fraction`` is the
    fraction of each sequence's KV pages kept in pinned host memory (its first
    pages).  ``max_ctx`` bounds the tokens a sequence can hold."""

    def __init__(self, shape: LlamaShape, *, batch: int, max_ctx: int, weight_offload: float = 0.0,
                 kv_host_fraction: float = 0.0, group=None, dtype=torch.float16, device="cuda",
                 fused_allreduce: bool = False):
        super().__init__()
        self.s = shape
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        G = self.world
        if shape.heads % G or shape.kv_heads % G or shape.ffn % G:
            raise ValueError(f"heads {shape.heads}, kv_heads {shape.kv_heads} and ffn {shape.ffn} must divide by {G}")
        if shape.head_dim != 128:
            raise ValueError("the decode attention kernel serves head_dim 128")
        self.hq, self.hkv, self.ffn_r = shape.heads // G, shape.kv_heads // G, shape.ffn // G
        self.vocab_r = vocab_rows_per_rank(shape.vocab, G)
        self.B, self.max_ctx, self.dtype, self.device = batch, max_ctx, dtype, device
        self.weight_offload = float(weight_offload)
        self.kv_host_fraction = float(kv_host_fraction)
        self.layers = nn.ModuleList()
        self.embed = None
        self.final_w = None
        self.lm_head = None
        self._alloc_kv()
        self._alloc_buffers()
        self.graph = None
        # o and down with their all-reduce fused: the row-parallel kernel leaves
        # its partial in place and the RMSNorm that follows reads the sum over
        # ranks through the NVSwitch multicast mapping.  Without multicast the
        # decoder keeps the NCCL all-reduce (measured faster than peer pushes).
        self.ar = None
        if fused_allreduce and self.world > 1:
            from .tp import SymmetricAllReduce

            ar = SymmetricAllReduce(batch * shape.hidden, group=group, dtype=dtype, consumer_reduces=True)
            self.ar = ar if ar.publish_only else None
        self.use_fused = self.ar is not None  # which reduction forward_step uses (see ``capture``)
        self.allreduce_times_ms = None

    # ------------------------------------------------------------- weights
    def _make_linear(self, w: torch.Tensor) -> nn.Module:
        from .tp import make_offloaded_shard

        return make_offloaded_shard(w, self.weight_offload)

    def _shard_layer(self, full: dict, l: int) -> dict:
        """This rank's slices of layer l's full weights (transformers names)."""
        s, r, d = self.s, self.rank, self.s.head_dim
        q = full["q"][r * self.hq * d:(r + 1) * self.hq * d]
        k = full["k"][r * self.hkv * d:(r + 1) * self.hkv * d]
        v = full["v"][r * self.hkv * d:(r + 1) * self.hkv * d]
        o = full["o"][:, r * self.hq * d:(r + 1) * self.hq * d]
        g = full["gate"][r * self.ffn_r:(r + 1) * self.ffn_r]
        u = full["up"][r * self.ffn_r:(r + 1) * self.ffn_r]
        dn = full["down"][:, r * self.ffn_r:(r + 1) * self.ffn_r]
        from .runtime import interleave_gate_up

        gate_up = interleave_gate_up(g, u) if self.fuse_glu else torch.cat([g, u], 0)
        return {"qkv": torch.cat([q, k, v], 0), "o": o, "gate_up": gate_up, "down": dn}

    @property
    def fuse_glu(self) -> bool:
        """gate_up's epilogue applies the SiLU gate when the rank's FFN width is a
        whole number of 16-feature blocks (gate and up rows interleaved)."""
        return self.__dict__.get("_fuse_glu", self.ffn_r % 16 == 0)

    @fuse_glu.setter
    def fuse_glu(self, on: bool) -> None:
        self.__dict__["_fuse_glu"] = bool(on)

    def split_gate_up(self, gu: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(gate, up) columns of x @ gate_up^T in this decoder's row order."""
        f = self.ffn_r
        if not self.fuse_glu:
            return gu[..., :f], gu[..., f:]
        blocks = gu.reshape(*gu.shape[:-1], f // 16, 2, 16)
        return blocks[..., 0, :].reshape(*gu.shape[:-1], f), blocks[..., 1, :].reshape(*gu.shape[:-1], f)

    def _add_layer(self, full: dict) -> None:
        sh = self._shard_layer(full, len(self.layers))
        mods = {n: self._make_linear(sh[n].to(self.device, self.dtype).contiguous()) for n in ("qkv", "o", "gate_up", "down")}
        self.layers.append(_Layer(mods["qkv"], mods["o"], mods["gate_up"], mods["down"],
                                  full["in_norm"].to(self.device, self.dtype), full["post_norm"].to(self.device, self.dtype)))

    def _set_head(self, embed: torch.Tensor, final_w: torch.Tensor, lm_head: torch.Tensor) -> None:
        self.embed = embed.to(self.device, self.dtype).contiguous()
        self.final_w = final_w.to(self.device, self.dtype)
        r, vr = self.rank, self.vocab_r
        shard = lm_head[r * vr:(r + 1) * vr].to(self.device, self.dtype)
        if shard.shape[0] < vr:  # the last rank's shard is padded with rows that never win
            shard = torch.cat([shard, torch.zeros(vr - shard.shape[0], shard.shape[1], dtype=shard.dtype,
                                                  device=shard.device)], 0)
        self.lm_head = self._make_linear(shard.contiguous())
        self.vocab_valid = max(0, min(vr, self.s.vocab - r * vr))

    @torch.no_grad()
    def load_hf(self, hf_model: nn.Module) -> "TPLlamaDecoder":
        """Shards the weights of a transformers LlamaForCausalLM onto this rank."""
        m = hf_model.model
        for layer in m.layers:
            at, mlp = layer.self_attn, layer.mlp
            self._add_layer({"q": at.q_proj.weight, "k": at.k_proj.weight, "v": at.v_proj.weight,
                             "o": at.o_proj.weight, "gate": mlp.gate_proj.weight, "up": mlp.up_proj.weight,
                             "down": mlp.down_proj.weight, "in_norm": layer.input_layernorm.weight,
                             "post_norm": layer.post_attention_layernorm.weight})
        self._set_head(m.embed_tokens.weight, m.norm.weight, hf_model.lm_head.weight)
        return self

    @torch.no_grad()
    def init_random(self, seed: int = 0, std: float = 0.02) -> "TPLlamaDecoder":
        """N(0, std) weights and unit norms.  Every rank draws the same full matrices
        from per-matrix seeds and keeps its shard, so the model does not depend on
        the tensor-parallel size."""
        s, dev = self.s, self.device
        h, d = s.hidden, s.head_dim

        def randn(shape, tag):
            g = torch.Generator(device=dev).manual_seed((seed * 1_000_003 + tag) % (2**63))
            return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std).to(self.dtype)

        ones = torch.ones(h, device=dev, dtype=self.dtype)
        for l in range(s.layers):
            t = 16 * (l + 1)
            self._add_layer({"q": randn((s.heads * d, h), t), "k": randn((s.kv_heads * d, h), t + 1),
                             "v": randn((s.kv_heads * d, h), t + 2), "o": randn((h, s.heads * d), t + 3),
                             "gate": randn((s.ffn, h), t + 4), "up": randn((s.ffn, h), t + 5),
                             "down": randn((h, s.ffn), t + 6), "in_norm": ones, "post_norm": ones})
        self._set_head(randn((s.vocab, h), 1), ones, randn((s.vocab, h), 2))
        torch.cuda.synchronize()
        return self

    # ------------------------------------------------------------------ KV
    def _alloc_kv(self) -> None:
        pages = -(-self.max_ctx // PAGE)
        n_host = int(round(self.kv_host_fraction * pages))
        n_host = min(pages, max(0, n_host))
        self.pages_per_seq, self.host_pages_per_seq = pages, n_host
        B, L, hkv, d = self.B, self.s.layers, self.hkv, self.s.head_dim
        dev_pages, host_pages = B * (pages - n_host), B * n_host
        self.kv_dev = (torch.empty(L, 2, dev_pages, hkv, PAGE, d, dtype=self.dtype, device=self.device)
                       if dev_pages else None)
        self.kv_host = (torch.empty(L, 2, host_pages, hkv, PAGE, d, dtype=self.dtype, pin_memory=True)
                        if host_pages else None)
        table = torch.empty(B, pages, dtype=torch.int32)
        for b in range(B):
            for j in range(pages):
                table[b, j] = (-1 - (b * n_host + j)) if j < n_host else b * (pages - n_host) + (j - n_host)
        self.block_table = table.to(self.device)
        self.split = auto_split_size(B, hkv, self.max_ctx)

    def kv_bytes(self) -> tuple[int, int]:
        """(host, device) bytes of this rank's KV pools."""
        hb = self.kv_host.numel() * self.kv_host.element_size() if self.kv_host is not None else 0
        db = self.kv_dev.numel() * self.kv_dev.element_size() if self.kv_dev is not None else 0
        return hb, db

    @torch.no_grad()
    def fill_kv_random(self, ctx: int, seed: int = 0) -> None:
        """Stands in for a prefill of ``ctx`` tokens per sequence: N(0, 1) K/V in every
        page, positions set so that the next decode step writes token ``ctx``."""
        g = torch.Generator(device=self.device).manual_seed(seed + 7 * self.rank)
        if self.kv_dev is not None:
            self.kv_dev.normal_(generator=g)
        if self.kv_host is not None:
            flat = self.kv_host.view(-1)
            chunk = 1 << 28
            for i in range(0, flat.numel(), chunk):
                n = min(chunk, flat.numel() - i)
                flat[i:i + n].copy_(torch.randn(n, generator=g, device=self.device, dtype=self.dtype))
        torch.cuda.synchronize()
        self.set_positions(ctx)

    def _pools(self, l: int):
        kd = self.kv_dev[l, 0] if self.kv_dev is not None else None
        vd = self.kv_dev[l, 1] if self.kv_dev is not None else None
        kh = self.kv_host[l, 0] if self.kv_host is not None else None
        vh = self.kv_host[l, 1] if self.kv_host is not None else None
        return kd, vd, kh, vh

    # ---------------------------------------------------------- decode step
    def _alloc_buffers(self) -> None:
        B, d = self.B, self.s.head_dim
        self.ids = torch.zeros(B, dtype=torch.long, device=self.device)
        self.pos = torch.zeros(B, dtype=torch.int32, device=self.device)
        self.seq_lens = torch.ones(B, dtype=torch.int32, device=self.device)
        self.attn_out = torch.empty(B, self.hq, d, dtype=self.dtype, device=self.device)
        ns = -(-self.max_ctx // auto_split_size(B, self.hkv, self.max_ctx))
        self.partial_o = torch.empty(B, self.hq, ns, d, dtype=torch.float32, device=self.device)
        self.partial_ml = torch.empty(B, self.hq, ns, 2, dtype=torch.float32, device=self.device)
        # The last split of each (sequence, KV head) merges in the attention
        # kernel; every call leaves these counters at zero.
        self.merge_counters = torch.zeros(B * self.hkv, dtype=torch.int32, device=self.device)
        self.inv_freq = 1.0 / (self.s.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32, device=self.device) / d))
        self.next_ids = torch.zeros(B, dtype=torch.long, device=self.device)
        self.logits_full = None
        h = self.s.hidden
        self.hidden = torch.empty(B, h, dtype=self.dtype, device=self.device)  # running residual stream
        self.x_buf = torch.empty(B, h, dtype=self.dtype, device=self.device)
        self.q_buf = torch.empty(B, self.hq, d, dtype=self.dtype, device=self.device)
        self.act_buf = torch.empty(B, self.ffn_r, dtype=self.dtype, device=self.device)
        self.o_buf = torch.empty(B, h, dtype=self.dtype, device=self.device)
        self.dn_buf = torch.empty(B, h, dtype=self.dtype, device=self.device)

    def set_positions(self, pos: int) -> None:
        self.pos.fill_(pos)

    def _all_reduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)

    def _add_norm(self, y: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """hidden += y (summed over ranks); returns RMSNorm(hidden) * w.  In
        publish-only mode the sum over ranks is read here, inside the norm."""
        from .decode_ops import rmsnorm

        if self.use_fused:
            return self.ar.rmsnorm(y, self.hidden, w, self.s.eps, self.x_buf)
        return rmsnorm(y, w, self.s.eps, residual=self.hidden, out=self.x_buf)

    def _row_parallel(self, mod: nn.Module, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """A row-parallel projection summed over the ranks: the fused kernel when
        enabled, else the local linear followed by an NCCL all-reduce."""
        if not self.use_fused:
            y = mod(x)
            self._all_reduce(y)
            return y
        from .runtime import linear_split

        wh, wd = self._tiers(mod)
        return linear_split(x, out, wh, wd, allreduce=self.ar)

    @staticmethod
    def _tiers(mod: nn.Module) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        """(host, device) transposed weights of an offloaded module, host rows first."""
        if hasattr(mod, "weight_h"):
            return (mod.weight_h if mod.out_features_h > 0 else None,
                    mod.weight_d if mod.out_features_d > 0 else None)
        return (None, mod.weight) if mod.weight.is_cuda else (mod.weight, None)

    def _gated(self, mod: nn.Module, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """silu(gate) * up straight from the gate_up kernel's epilogue."""
        from .runtime import linear_split

        wh, wd = self._tiers(mod)
        return linear_split(x, out, wh, wd, glu=True)

    def forward_step(self, keep_logits: bool = False) -> torch.Tensor:
        """One decode step on the static buffers: embeds ``ids`` at ``pos``, writes
        their K/V, and leaves the greedy tokens in ``next_ids``; advances nothing.
        Per layer: RMSNorm (residual add fused), qkv, rotary and KV append (one
        kernel), attention, o + all-reduce, RMSNorm, gate_up with the SiLU gate in
        its epilogue (or gate_up, then SiLU-gate), down + all-reduce."""
        from .decode_ops import rmsnorm, silu_mul

        s, B, d = self.s, self.B, self.s.head_dim
        t = self._span
        with t("embed"):
            torch.add(self.pos, 1, out=self.seq_lens)
            self.hidden.copy_(self.embed[self.ids])
        qd = self.hq * d
        scale = 1.0 / math.sqrt(d)
        with t("norm"):
            x = rmsnorm(self.hidden, self.layers[0].in_w, s.eps, out=self.x_buf)
        for l, layer in enumerate(self.layers):
            with t("qkv"):
                qkv = layer.qkv(x)
            kdev, vdev, khost, vhost = self._pools(l)
            with t("rope+kv_append"):
                rope_kv_append(qkv, self.pos, self.inv_freq, self.hq, self.hkv, d, self.q_buf, kdev, vdev, khost,
                               vhost, self.block_table)
            with t("attention"):
                decode_paged(self.q_buf, kdev, vdev, khost, vhost, self.block_table, self.seq_lens, scale,
                             self.split, out=self.attn_out, partial_o=self.partial_o, partial_ml=self.partial_ml,
                             max_seq_len=self.max_ctx, merge_counters=self.merge_counters)
            with t("o" if self.use_fused else "o+allreduce"):
                o = self._row_parallel(layer.o, self.attn_out.view(B, qd), self.o_buf)
            with t("allreduce+norm" if self.use_fused else "norm"):
                x = self._add_norm(o, layer.post_w)
            if self.fuse_glu:
                with t("gate_up+silu"):
                    act = self._gated(layer.gate_up, x, self.act_buf)
            else:
                with t("gate_up"):
                    gu = layer.gate_up(x)
                with t("silu"):
                    act = silu_mul(gu, out=self.act_buf)
            with t("down" if self.use_fused else "down+allreduce"):
                dn = self._row_parallel(layer.down, act, self.dn_buf)
            nxt_w = self.layers[l + 1].in_w if l + 1 < len(self.layers) else self.final_w
            with t("allreduce+norm" if self.use_fused else "norm"):
                x = self._add_norm(dn, nxt_w)
        with t("lm_head"):
            logits = self.lm_head(x)[:, :max(1, self.vocab_valid)]
        with t("pick"):
            val, idx = logits.float().max(dim=-1)
            if self.world > 1:
                pair = torch.stack([val, (idx + self.rank * self.vocab_r).float()], dim=-1)  # [B, 2]
                allp = torch.empty(self.world, B, 2, dtype=pair.dtype, device=pair.device)
                dist.all_gather_into_tensor(allp, pair, group=self.group)
                best = allp[:, :, 0].argmax(dim=0)  # first maximum, as argmax over the full row
                self.next_ids.copy_(allp[best, torch.arange(B, device=pair.device), 1].long())
            else:
                self.next_ids.copy_(idx)
        if keep_logits:
            if self.world > 1:
                parts = torch.empty(self.world * B, self.vocab_r, dtype=logits.dtype, device=logits.device)
                padded = torch.zeros(B, self.vocab_r, dtype=logits.dtype, device=logits.device)
                padded[:, :logits.shape[1]] = logits
                dist.all_gather_into_tensor(parts, padded, group=self.group)
                full = parts.view(self.world, B, self.vocab_r).permute(1, 0, 2).reshape(B, -1)
                self.logits_full = full[:, :s.vocab]
            else:
                self.logits_full = logits
        return self.next_ids

    def _span(self, name: str):
        """Timing scope of one op group of ``forward_step``: CUDA events around it
        while ``profile_step`` runs, nothing otherwise (graph capture included)."""
        timer = getattr(self, "_timer", None)
        return timer(name) if timer is not None else contextlib.nullcontext()

    @torch.inference_mode()
    def profile_step(self) -> dict[str, float]:
        """One eager decode step (plus the advance) with CUDA events around every op
        group; returns milliseconds per group summed over the layers.  Events
        between the kernels stop them from overlapping, so the sum exceeds a
        graph replay's time; the shares show where a step goes."""
        events = []

        @contextlib.contextmanager
        def timer(name):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            yield
            e1.record()
            events.append((name, e0, e1))

        self._timer = timer
        try:
            self.forward_step()
            self.advance()
        finally:
            self._timer = None
        torch.cuda.synchronize()
        out: dict[str, float] = {}
        for name, e0, e1 in events:
            out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
        return {k: round(v, 4) for k, v in out.items()}

    def kernel_launches_per_step(self) -> int:
        """Launches of this library's kernels in one ``forward_step``: the first
        RMSNorm; per layer the four linears (gate_up also applies the SiLU gate
        when ``fuse_glu``, else a SiLU-gate kernel follows), rotary with the KV
        append, attention (which also merges its splits) and two RMSNorms; then
        lm_head.  The torch ops around them (embedding gather, greedy pick) and
        NCCL's kernels are not counted."""
        return 1 + len(self.layers) * (8 if self.fuse_glu else 9) + 1

    def advance(self) -> None:
        """Feeds the greedy tokens back and moves every sequence one position on."""
        self.ids.copy_(self.next_ids)
        self.pos.add_(1)

    @torch.inference_mode()
    def capture(self, choose_allreduce: bool = False, trials: int = 5) -> None:
        """Captures one decode step plus the advance into a CUDA graph (after a warm-up
        step whose KV writes and advance are undone).

        With ``choose_allreduce`` and the fused reduction available, the step is
        captured both ways (consumer-side reduction, and linear + NCCL), each graph
        is replayed ``trials`` times from the same position, and the one whose
        slowest rank is faster is kept: which wins depends on the group size and
        the box.  Every rank captures and replays both graphs in the same order.
        ``allreduce_times_ms`` records the median replay time of each."""
        pos0, ids0 = self.pos.clone(), self.ids.clone()

        def one_graph():
            self.forward_step()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.forward_step()
                self.advance()
            self.pos.copy_(pos0)
            self.ids.copy_(ids0)
            torch.cuda.synchronize()
            return g

        if not (choose_allreduce and self.ar is not None and self.world > 1):
            self.graph = one_graph()
            return
        stream = torch.cuda.current_stream()
        graphs, times = {}, {}
        for fused in (True, False):
            self.use_fused = fused
            g = one_graph()
            ms = []
            for _ in range(trials + 1):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
                self.pos.copy_(pos0)  # every trial runs from the same position
                self.ids.copy_(ids0)
                torch.cuda.synchronize()
                ms.append(e0.elapsed_time(e1))
            graphs[fused] = g
            times[fused] = sorted(ms[1:])[len(ms[1:]) // 2]
        t = torch.tensor([times[True], times[False]], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        self.allreduce_times_ms = {"fused": float(t[0]), "nccl": float(t[1])}
        self.use_fused = bool(t[0] <= t[1])
        self.graph = graphs[self.use_fused]
        graphs.clear()  # the other graph (it may hold NCCL work) goes now
        torch.cuda.synchronize()

    def step(self) -> None:
        """One decode step + advance: a graph replay when captured."""
        if self.graph is not None:
            self.graph.replay()
        else:
            with torch.inference_mode():
                self.forward_step()
                self.advance()

    def release(self) -> None:
        """Drops the CUDA graph (it holds NCCL work) before the process group goes away."""
        self.graph = None
