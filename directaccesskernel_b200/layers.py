"""Offloaded Linear modules, mirroring app/python/layers/linearLayer.py and
app/python/layers/linearLayerMulticast.py of the reference.

Same classes, constructor arguments, attributes and methods:
``Linear`` (whole weight in one tier), ``LinearHorizontal`` (rows split between
pinned host memory and HBM), ``LinearMulticast`` / ``LinearHorizontalMulticast``
(the batched-decode / prefill variants).  Weights are kept transposed,
``[in_features, out_features]``, as the reference stores them, and each forward
runs one launch of the sm_100a split kernel on the current stream.

Differences from the reference, none of which change results:
  * the output is allocated with ``torch.empty``; the kernels write every
    element once (the reference zero-fills because it reduce-adds);
  * ``horizontal_split_weight`` accepts ``host_side="last"`` to keep the last
    rows on the host instead of the first (the output is identical);
  * the multicast classes accept ``h_m == d_m == 0`` (split from the ratio)
    and any token count; they run on the tcgen05 kernel, without multicast.
"""
from __future__ import annotations

import math

import torch
from torch import Tensor
from torch.nn import Module, Parameter, init

from . import runtime
from .config import TILE_K, TILE_K_MULTICAST, TILE_M, TILE_M_MULTICAST, TILE_N, TILE_N_MULTICAST
from .utils import build_tma_wgmma_k, build_tma_wgmma_mn, split_horizontal


def _blocked_ok(w: Tensor) -> bool:
    """Whether the reference's blocked ("debug") descriptor form covers all of ``w``."""
    return w.shape[0] % 8 == 0 and w.shape[1] % 64 == 0


def _pinned_empty(rows: int, cols: int, dtype: torch.dtype) -> Tensor:
    return torch.empty(rows, cols, dtype=dtype, device="cpu", pin_memory=True).contiguous()


class _OffloadLinearBase(Module):
    __constants__ = ["in_features", "out_features"]
    in_features: int
    out_features: int

    def __init__(self, in_features: int, out_features: int, smem_size: int, num_copy_blocks: int,
                 bias: bool = False, device=None, dtype=None, skip_init: bool = False) -> None:
        factory_kwargs = {"device": device, "dtype": dtype}
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.smem_size = smem_size
        self.num_copy_blocks = num_copy_blocks
        self.weight = Parameter(torch.empty((out_features, in_features), **factory_kwargs))
        if bias:
            self.bias = Parameter(torch.empty(out_features, **factory_kwargs))
        else:
            self.register_parameter("bias", None)
        if not skip_init:
            self.reset_parameters()
        self.output = None
        self.output_shape = None
        self.input_shape = None
        self.input_desc = None
        self.output_desc = None

    def reset_parameters(self) -> None:
        """linearLayer.py:59-70: kaiming-uniform weight, uniform bias."""
        init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in, _ = init._calculate_fan_in_and_fan_out(self.weight)
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            init.uniform_(self.bias, -bound, bound)

    def _io_descs(self, input: Tensor, tile_k: int, tile_n: int, tile_m: int, debug: bool) -> Tensor:
        """Input/output descriptors, rebuilt on shape change and re-pointed otherwise
        (linearLayer.py:103-118)."""
        x2 = input.reshape(-1, self.in_features)
        if x2.stride(-1) != 1 or x2.stride(0) != self.in_features:
            x2 = x2.contiguous()
        # The blocked (debug) output form only covers whole groups of 8 rows.
        debug = debug and x2.shape[0] % 8 == 0
        if self.input_desc is None or self.input_shape != input.shape:
            self.input_shape = input.shape
            _, self.input_desc = build_tma_wgmma_k(x2, tile_k, tile_n)
        else:
            runtime.tensormap_replace_address(self.input_desc, x2)
        expected_output_shape = input.shape[:-1] + (self.out_features,)
        output = torch.empty(*expected_output_shape, device=input.device, dtype=input.dtype)
        if self.output_desc is None or self.output_shape != expected_output_shape:
            self.output_shape = output.shape
            _, self.output_desc = build_tma_wgmma_mn(output.view(-1, self.out_features), tile_m, tile_n, debug=debug)
        else:
            runtime.tensormap_replace_address(self.output_desc, output)
        return output

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


class _SingleTierMixin:
    def move_weight_to_device(self, device):
        """linearLayer.py:72-80: transposed weight to pinned host ("cpu") or HBM."""
        if device == "cpu":
            weight_h = _pinned_empty(self.in_features, self.out_features, torch.float16
                                     if self.weight.dtype not in (torch.float16, torch.bfloat16) else self.weight.dtype)
        else:
            dt = self.weight.dtype if self.weight.dtype in (torch.float16, torch.bfloat16) else torch.float16
            weight_h = torch.empty(self.in_features, self.out_features, dtype=dt, device="cuda")
        weight_h.copy_(self.weight.data.T, non_blocking=False)
        del self.weight
        self.weight = None
        self.weight = Parameter(weight_h, requires_grad=False)

    def config(self, num_blocks: int, sms_per_row: int):
        """linearLayer.py:87-89."""
        self.num_copy_blocks = num_blocks
        self.sms_per_row = sms_per_row


class Linear(_SingleTierMixin, _OffloadLinearBase):
    """app/python/layers/linearLayer.py:14-139: whole weight in one tier."""

    def __init__(self, in_features, out_features, smem_size, num_copy_blocks, bias=False, device=None,
                 dtype=None, skip_init=False):
        super().__init__(in_features, out_features, smem_size, num_copy_blocks, bias, device, dtype, skip_init)
        self.sms_per_row = 1
        self.w_desc = None

    def build_tma_desc(self):
        if self.w_desc is None:
            _, self.w_desc = build_tma_wgmma_mn(self.weight, TILE_M, TILE_K)

    def forward(self, input: Tensor) -> Tensor:
        self.build_tma_desc()
        output = self._io_descs(input, TILE_K, TILE_N, TILE_M, debug=False)
        runtime.gemv(self.w_desc, self.input_desc, self.output_desc, self.out_features, input.shape[:-1].numel(),
                     self.in_features, self.num_copy_blocks, self.smem_size, self.sms_per_row)
        if self.bias is not None:
            output += self.bias
        return output


class _HorizontalMixin:
    def _split(self, offload: float, num_blocks: int, num_host_blocks: int, h_sms_per_row: int,
               d_sms_per_row: int, h_m: int, d_m: int, host_side: str) -> None:
        """linearLayer.py:207-246: [0:h_m) rows to pinned host memory, the rest to HBM,
        both stored transposed.  ``host_side="last"`` keeps the last h_m rows on host."""
        if host_side not in ("first", "last"):
            raise ValueError(f"host_side must be 'first' or 'last', got {host_side!r}")
        self.num_copy_blocks = num_blocks
        self.num_copy_blocks_host = num_host_blocks
        self.h_sms_per_row = h_sms_per_row
        self.d_sms_per_row = d_sms_per_row
        if h_m == 0 and d_m == 0:
            self.out_features_h, self.out_features_d = split_horizontal((self.out_features, self.in_features), offload)
        else:
            self.out_features_h = h_m
            self.out_features_d = d_m
        if self.out_features_h + self.out_features_d != self.out_features:
            raise ValueError(f"h_m + d_m = {self.out_features_h + self.out_features_d} != out_features {self.out_features}")
        self.host_side = host_side
        dt = self.weight.dtype if self.weight.dtype in (torch.float16, torch.bfloat16) else torch.float16
        w = self.weight.data
        if host_side == "first":
            host_rows, dev_rows = w[: self.out_features_h, :], w[self.out_features_h:, :]
        else:
            host_rows, dev_rows = w[self.out_features_d:, :], w[: self.out_features_d, :]
        weight_h = _pinned_empty(self.in_features, self.out_features_h, dt)
        weight_d = torch.empty(self.in_features, self.out_features_d, dtype=dt, device="cuda")
        weight_h.copy_(host_rows.T, non_blocking=False)
        weight_d.copy_(dev_rows.T, non_blocking=False)
        self.weight_h = Parameter(weight_h, requires_grad=False)
        self.weight_d = Parameter(weight_d, requires_grad=False)
        del self.weight
        self.weight = None

    def set_blocks(self, num_blocks: int, num_host_blocks: int):
        """linearLayerMulticast.py:221-223."""
        self.num_copy_blocks = num_blocks
        self.num_copy_blocks_host = num_host_blocks

    def _forward_split(self, input: Tensor, tile_k: int, tile_n: int, tile_m: int, debug: bool, launch) -> Tensor:
        if getattr(self, "host_side", "first") == "last":
            x2 = input.reshape(-1, self.in_features)
            if x2.stride(-1) != 1:
                x2 = x2.contiguous()
            output = torch.empty(*input.shape[:-1], self.out_features, device=input.device, dtype=input.dtype)
            runtime.linear_split(
                x2, output.view(-1, self.out_features),
                self.weight_h if self.out_features_h > 0 else None,
                self.weight_d if self.out_features_d > 0 else None,
                host_col_offset=self.out_features_d, dev_col_offset=0,
                host_ctas=self.num_copy_blocks_host if self.num_copy_blocks > 0 else 0,
                dev_ctas=self.num_copy_blocks - self.num_copy_blocks_host if self.num_copy_blocks > 0 else 0,
                host_ksplit=self.h_sms_per_row, dev_ksplit=self.d_sms_per_row)
        else:
            self.build_tma_desc()
            output = self._io_descs(input, tile_k, tile_n, tile_m, debug)
            launch(self.w_desc_h, self.w_desc_d, self.input_desc, self.output_desc, self.out_features_h,
                   self.out_features_d, input.shape[:-1].numel(), self.in_features, self.num_copy_blocks,
                   self.num_copy_blocks_host, self.smem_size, self.h_sms_per_row, self.d_sms_per_row)
        if self.bias is not None:
            output += self.bias
        return output


class LinearHorizontal(_HorizontalMixin, _OffloadLinearBase):
    """app/python/layers/linearLayer.py:142-341: rows split between host and HBM."""

    def __init__(self, in_features, out_features, smem_size, num_copy_blocks, bias=False, device=None,
                 dtype=None, skip_init=False):
        super().__init__(in_features, out_features, smem_size, num_copy_blocks, bias, device, dtype, skip_init)
        self.h_sms_per_row = 1
        self.d_sms_per_row = 1
        self.num_copy_blocks_host = 0
        self.w_desc_h = None
        self.w_desc_d = None

    def horizontal_split_weight(self, offload: float, num_blocks: int, num_host_blocks: int, h_sms_per_row: int,
                                d_sms_per_row: int, h_m: int = 0, d_m: int = 0, host_side: str = "first") -> None:
        self._split(offload, num_blocks, num_host_blocks, h_sms_per_row, d_sms_per_row, h_m, d_m, host_side)

    def build_tma_desc(self):
        if self.w_desc_h is None and self.out_features_h > 0:
            _, self.w_desc_h = build_tma_wgmma_mn(self.weight_h, TILE_M, TILE_K)
        if self.w_desc_d is None and self.out_features_d > 0:
            _, self.w_desc_d = build_tma_wgmma_mn(self.weight_d, TILE_M, TILE_K)

    def forward_naieve(self, input: Tensor) -> Tensor:
        """linearLayer.py:269-291: same result, descriptors rebuilt on every call."""
        self.input_desc = self.output_desc = None
        return self.forward(input)

    def forward(self, input: Tensor) -> Tensor:
        return self._forward_split(input, TILE_K, TILE_N, TILE_M, False, runtime.gemv_horizontal)


class LinearMulticast(_SingleTierMixin, _OffloadLinearBase):
    """app/python/layers/linearLayerMulticast.py:14-136 (tcgen05, no multicast)."""

    def __init__(self, in_features, out_features, smem_size, num_copy_blocks, bias=False, device=None,
                 dtype=None, skip_init=False):
        super().__init__(in_features, out_features, smem_size, num_copy_blocks, bias, device, dtype, skip_init)
        self.sms_per_row = 1
        self.w_desc = None
        self.prefill = True

    def build_tma_desc(self):
        if self.w_desc is None:
            _, self.w_desc = build_tma_wgmma_mn(self.weight, TILE_M_MULTICAST, TILE_K_MULTICAST,
                                                debug=_blocked_ok(self.weight))

    def forward(self, input: Tensor) -> Tensor:
        self.build_tma_desc()
        output = self._io_descs(input, TILE_K_MULTICAST, TILE_N_MULTICAST, TILE_M_MULTICAST, debug=True)
        launch = runtime.gemv_multicast_prefill if self.prefill else runtime.gemv_multicast
        blocks = 0 if self.prefill else self.num_copy_blocks
        launch(self.w_desc, self.input_desc, self.output_desc, self.out_features, input.shape[:-1].numel(),
               self.in_features, blocks, self.smem_size, self.sms_per_row)
        if self.bias is not None:
            output += self.bias
        return output


class LinearHorizontalMulticast(_HorizontalMixin, _OffloadLinearBase):
    """app/python/layers/linearLayerMulticast.py:140-312 (tcgen05, no multicast)."""

    def __init__(self, in_features, out_features, smem_size, num_copy_blocks, bias=False, device=None,
                 dtype=None, skip_init=False):
        super().__init__(in_features, out_features, smem_size, num_copy_blocks, bias, device, dtype, skip_init)
        self.h_sms_per_row = 1
        self.d_sms_per_row = 1
        self.num_copy_blocks_host = 0
        self.w_desc_h = None
        self.w_desc_d = None
        self.prefill = True

    def horizontal_split_weight(self, offload: float, num_blocks: int, num_host_blocks: int, h_sms_per_row: int,
                                d_sms_per_row: int, h_m: int = 0, d_m: int = 0, host_side: str = "first") -> None:
        self._split(offload, num_blocks, num_host_blocks, h_sms_per_row, d_sms_per_row, h_m, d_m, host_side)

    def build_tma_desc(self):
        if self.w_desc_h is None and self.out_features_h > 0:
            _, self.w_desc_h = build_tma_wgmma_mn(self.weight_h, TILE_M_MULTICAST, TILE_K_MULTICAST,
                                                  debug=_blocked_ok(self.weight_h))
        if self.w_desc_d is None and self.out_features_d > 0:
            _, self.w_desc_d = build_tma_wgmma_mn(self.weight_d, TILE_M_MULTICAST, TILE_K_MULTICAST,
                                                  debug=_blocked_ok(self.weight_d))

    def forward_naieve(self, input: Tensor) -> Tensor:
        self.input_desc = self.output_desc = None
        return self.forward(input)

    def forward(self, input: Tensor) -> Tensor:
        if self.prefill:
            # The reference's prefill path hard-codes 128 CTAs, 64 of them on host rows
            # (linearLayerMulticast.py:296-297); the B200 schedule picks its own.
            def launch(a_h, a_d, b, c, h_M, d_M, N, K, _blocks, _host_blocks, smem, h_spr, d_spr):
                runtime.gemv_horizontal_multicast_prefill(a_h, a_d, b, c, h_M, d_M, N, K, 0, 0, smem, h_spr, d_spr)
        else:
            launch = runtime.gemv_horizontal_multicast
        return self._forward_split(input, TILE_K_MULTICAST, TILE_N_MULTICAST, TILE_M_MULTICAST, True, launch)
