"""Tensor-parallel offloaded linear layers for one 8xB200 box.

The reference has no multi-GPU code.  These layers shard a linear layer
Megatron-style over a torch.distributed process group (NCCL over NVLink on the
GPUs, gloo in the CPU tests):
  * ColumnParallelLinear: rank r owns output features [r*N/G, (r+1)*N/G); the
    local result is all-gathered when ``gather_output`` (q/k/v, gate/up and
    lm_head keep it sharded);
  * RowParallelLinear: rank r owns input features [r*K/G, (r+1)*K/G) and
    consumes the matching slice of its input; the partial products are summed
    with one all-reduce (o and down projections).
Each rank's shard is an ordinary offloaded module (LinearHorizontal and
friends), split between that GPU's HBM and pinned host memory on the GPU's own
NUMA node, so every GPU streams its own host rows over its own host link.  The
collectives run on the current stream after the local kernel.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
from torch import nn


def shard_rows(weight: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Output-feature shard [N/G, K] of an nn.Linear weight [N, K]."""
    n = weight.shape[0]
    if n % world:
        raise ValueError(f"out_features {n} is not divisible by the tensor-parallel size {world}")
    step = n // world
    return weight[rank * step:(rank + 1) * step]


def shard_cols(weight: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Input-feature shard [N, K/G] of an nn.Linear weight [N, K]."""
    k = weight.shape[1]
    if k % world:
        raise ValueError(f"in_features {k} is not divisible by the tensor-parallel size {world}")
    step = k // world
    return weight[:, rank * step:(rank + 1) * step]


def _group_info(group):
    return dist.get_rank(group), dist.get_world_size(group)


class ColumnParallelLinear(nn.Module):
    """y = x W^T with W's rows sharded; ``local`` computes x W_r^T for this rank."""

    def __init__(self, local: nn.Module, out_features: int, group=None, gather_output: bool = True):
        super().__init__()
        self.local = local
        self.group = group
        self.out_features = out_features
        self.gather_output = gather_output
        self.rank, self.world = _group_info(group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.local(x)
        if not self.gather_output or self.world == 1:
            return y
        y2 = y.reshape(-1, y.shape[-1]).contiguous()
        parts = torch.empty((self.world * y2.shape[0], y2.shape[1]), dtype=y.dtype, device=y.device)
        dist.all_gather_into_tensor(parts, y2, group=self.group)
        # [G * rows, N/G] -> [rows, N]: shard r holds output features r*N/G .. (r+1)*N/G.
        full = parts.view(self.world, y2.shape[0], y2.shape[1]).permute(1, 0, 2).reshape(y2.shape[0], -1)
        return full.reshape(*y.shape[:-1], self.out_features)


class RowParallelLinear(nn.Module):
    """y = x W^T with W's columns sharded; partial products summed by all-reduce."""

    def __init__(self, local: nn.Module, in_features: int, group=None, input_is_parallel: bool = False):
        super().__init__()
        self.local = local
        self.group = group
        self.in_features = in_features
        self.input_is_parallel = input_is_parallel
        self.rank, self.world = _group_info(group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.input_is_parallel and self.world > 1:
            step = self.in_features // self.world
            x = x[..., self.rank * step:(self.rank + 1) * step].contiguous()
        y = self.local(x)
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        return y


def make_offloaded_shard(weight_shard: torch.Tensor, offload_ratio: float, *, host_side: str = "first",
                         device: str | torch.device = "cuda") -> nn.Module:
    """An offloaded module holding ``weight_shard`` ([N_r, K_r]): LinearHorizontal
    for 0 < r < 1, a single-tier Linear in HBM (r = 0) or pinned host memory (r = 1)."""
    from .layers import Linear, LinearHorizontal
    from .utils import get_smem_size, split_horizontal

    n, k = weight_shard.shape
    dt = weight_shard.dtype if weight_shard.dtype in (torch.float16, torch.bfloat16) else torch.float16
    if 0.0 < offload_ratio < 1.0:
        # A small shard may round to no host rows, or to all of them (rows move
        # in 64-row boxes): it is then a single-tier module.
        h_m, d_m = split_horizontal((n, k), offload_ratio)
        if h_m == 0 or d_m == 0:
            offload_ratio = 1.0 if h_m else 0.0
    if 0.0 < offload_ratio < 1.0:
        mod = LinearHorizontal(k, n, get_smem_size(), 0, device=device, dtype=dt, skip_init=True)
        with torch.no_grad():
            mod.weight.copy_(weight_shard)
        mod.horizontal_split_weight(offload_ratio, 0, 0, 1, 1, host_side=host_side)
    else:
        mod = Linear(k, n, get_smem_size(), 0, device=device, dtype=dt, skip_init=True)
        with torch.no_grad():
            mod.weight.copy_(weight_shard)
        mod.move_weight_to_device("cpu" if offload_ratio >= 1.0 else "cuda")
    mod.build_tma_desc()
    return mod


class SymmetricAllReduce:
    """Buffers for the all-reduce fused into the linear kernel
    (``dak_linear_split_allreduce``), in torch symmetric memory (mapped into
    every rank of ``group``), plus this rank's call counters.

    Two modes, chosen collectively: "multimem" when the allocation has a
    multicast mapping (NVSwitch): each rank keeps its FP32 partials in its own
    buffer and reads the sum with multimem.ld_reduce; otherwise "peer": each
    rank pushes its 16-bit partials into every rank's receive slots.  One
    instance serves any number of sequential calls on one stream; every rank
    must make the same calls in the same order."""

    MAX_CTAS = 1024

    def __init__(self, slot_elems: int, group=None, dtype=torch.float16, timeout_us: int = 2_000_000,
                 multicast: bool = True, consumer_reduces: bool = False):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        name = self.group.group_name
        self.rank, self.world = _group_info(self.group)
        if self.world > 8:
            raise ValueError("the fused all-reduce serves at most 8 ranks")
        self.slot_elems = int(slot_elems)
        self.flags = symm_mem.empty(self.MAX_CTAS * self.world, dtype=torch.int32, device="cuda")
        self.flags.zero_()
        self.mode, self.own, self.mc = "peer", None, 0
        if multicast:
            own = symm_mem.empty(2 * self.slot_elems, dtype=torch.float32, device="cuda")
            own.zero_()
            torch.cuda.synchronize()
            h = symm_mem.rendezvous(own, name)
            try:
                has = bool(symm_mem._SymmetricMemory.has_multicast_support(
                    symm_mem.DeviceType.CUDA, torch.cuda.current_device()))
            except (AttributeError, TypeError, RuntimeError):
                has = False
            ok = torch.tensor([1 if (has and h.multicast_ptr) else 0], dtype=torch.int32, device="cuda")
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
            if int(ok.item()):
                self.mode, self.own, self._hm = "multimem", own, h
                self.mc = h.multicast_ptr + (own.data_ptr() - h.buffer_ptrs[self.rank])
        self.buf = None
        if self.mode == "peer":
            self.buf = symm_mem.empty(2 * self.world * self.slot_elems, dtype=dtype, device="cuda")
            torch.cuda.synchronize()
            self._hb = symm_mem.rendezvous(self.buf, name)
        torch.cuda.synchronize()
        self._hf = symm_mem.rendezvous(self.flags, name)
        self.counters = torch.zeros(2, dtype=torch.int32, device="cuda")  # epoch, done
        dist.barrier(group=self.group)
        self.timeout_us = int(timeout_us)
        # Publish-only (multimem mode): the linear kernel leaves its partials in
        # place and the consumer, ``rmsnorm``, reads their sum.
        self.publish_only = bool(consumer_reduces and self.mode == "multimem")
        self._args = None

    @staticmethod
    def _peer_ptrs(h, t, rank):
        off = t.data_ptr() - h.buffer_ptrs[rank]
        return [p + off for p in h.buffer_ptrs]

    def args(self, y: torch.Tensor):
        from . import _lib

        if y.shape[0] * y.stride(0) > self.slot_elems:
            raise RuntimeError(f"output of {y.shape[0]} x {y.stride(0)} exceeds the slots of {self.slot_elems}")
        if self._args is None:
            a = _lib.AllReduceArgs()
            a.world, a.rank = self.world, self.rank
            flags = self._peer_ptrs(self._hf, self.flags, self.rank)
            bufs = self._peer_ptrs(self._hb, self.buf, self.rank) if self.mode == "peer" else [0] * self.world
            for r in range(self.world):
                a.buffers[r] = bufs[r] or None
                a.flags[r] = flags[r]
            a.slot_elems = self.slot_elems
            a.epoch = self.counters.data_ptr()
            a.done = self.counters.data_ptr() + 4
            a.timeout_us = self.timeout_us
            if self.mode == "multimem":
                a.own_f32, a.mc_f32 = self.own.data_ptr(), self.mc
            a.publish_only = 1 if self.publish_only else 0
            self._args = a
        return self._args

    def rmsnorm(self, y: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                out: torch.Tensor) -> torch.Tensor:
        """After a publish-only linear call that targeted ``y`` (not written): residual
        += the sum over ranks (rounded to 16 bit), out = RMSNorm(residual) * weight."""
        from ._lib import LIB, check
        from .runtime import dak_dtype

        if not self.publish_only:
            raise RuntimeError("rmsnorm of the all-reduce needs the publish-only (multimem) mode")
        rows, cols = residual.shape
        if not (residual.is_contiguous() and out.is_contiguous() and weight.numel() == cols):
            raise RuntimeError("residual and out must be contiguous [rows, cols], weight [cols]")
        check(LIB.dak_rmsnorm_allreduce(ctypes.byref(self.args(y)), residual.data_ptr(),
                                        weight.data_ptr(), out.data_ptr(), rows, cols, y.stride(0), float(eps),
                                        dak_dtype(residual.dtype), torch.cuda.current_stream().cuda_stream),
              "rmsnorm_allreduce")
        return out
