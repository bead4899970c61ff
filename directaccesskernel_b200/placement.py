"""Placement entry point, mirroring app/python/placement.py:1-212.

``place_model`` keeps the reference's signature, tables, errors and return
value.  B200 additions:
  * ``gpu_name="B200"`` (the default) uses the automatic schedule of the C ABI
    (``num_copy_blocks = 0``): host-tier CTAs sized to saturate the host link,
    the remaining SMs on the HBM tier, split-K chosen per shape;
  * ``hbm_budget_bytes=`` derives the offload ratio from an HBM budget instead
    of taking it from the caller (the reference has no budget API);
  * ``host_side="last"`` keeps the last rows of each weight on the host.
"""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

import torch
from torch import nn

DEFAULT_HORIZONTAL_CONFIG = {
    "GH200": {
        (7168, 7168): (2560, 4608, 40, 90, 1, 1),
        (7168, 28672): (2560, 4608, 40, 90, 1, 1),
        (28672, 7168): (10240, 18432, 40, 90, 1, 1),
    },
    "RTX6000": {
        (7168, 7168): (128, 7040, 2, 128, 1, 1),
        (7168, 28672): (192, 6976, 3, 128, 1, 1),
        (28672, 7168): (832, 27840, 8, 160, 1, 1),
        (4096, 4096): (64, 4032, 2, 128, 2, 2),
        (4096, 16384): (64, 4032, 2, 128, 2, 2),
        (16384, 4096): (384, 16000, 3, 140, 1, 1),
    },
    "B200": {},
}

# (h_m, d_m, h_blocks, d_blocks, h_sms_per_row, d_sms_per_row); zeros = split
# from the ratio and let the B200 schedule choose CTAs and split-K.
B200_DEFAULT_SPLIT = (0, 0, 0, 0, 1, 1)


@dataclass(frozen=True)
class ModelPlacementStats:
    host_bytes: int
    device_bytes: int
    actual_offload_ratio: float


def place_model(
    model: nn.Module,
    offload_ratio: float | None = None,
    *,
    gpu_name: str = "B200",
    use_config: bool = False,
    horizontal_config: Mapping[str, Mapping[tuple[int, int], tuple[int, int, int, int, int, int]]] | None = None,
    default_horizontal_config: Mapping[str, tuple[int, int, int, int, int, int]] | None = None,
    device: torch.device | str = "cuda",
    build_tma_desc: bool = True,
    hbm_budget_bytes: int | None = None,
    host_side: str = "first",
) -> ModelPlacementStats:
    """placement.py:35-75: non-custom tensors to the GPU, replaced linears split
    between host and HBM by ``offload_ratio`` (or by ``hbm_budget_bytes``)."""
    custom_types = _custom_linear_types()
    budget_mode = hbm_budget_bytes is not None
    if budget_mode:
        offload_ratio = offload_ratio_for_budget(model, hbm_budget_bytes)
    if offload_ratio is None:
        raise TypeError("place_model needs offload_ratio or hbm_budget_bytes")

    _move_non_custom_direct_tensors(model, custom_types, device)

    for name, module in model.named_modules():
        if not isinstance(module, custom_types):
            continue
        if _is_horizontal_linear(module):
            _place_horizontal_linear(
                name, module, offload_ratio, gpu_name=gpu_name, use_config=use_config,
                horizontal_config=horizontal_config or DEFAULT_HORIZONTAL_CONFIG,
                default_horizontal_config=default_horizontal_config, allow_edges=budget_mode,
                host_side=host_side,
            )
            _move_custom_linear_bias(module, device)
        elif _is_host_linear(module):
            target = "cpu" if offload_ratio >= 1.0 else device
            module.move_weight_to_device(target)
            _move_custom_linear_bias(module, device)
            if gpu_name == "B200":
                module.num_copy_blocks = 0
            if build_tma_desc:
                module.build_tma_desc()
        else:
            raise TypeError(f"Unsupported replaced Linear module at {name}: {type(module)!r}")
    return get_model_placement_stats(model)


def set_linear_prefill(model: nn.Module, prefill: bool) -> None:
    """placement.py:78-81."""
    for module in model.modules():
        if hasattr(module, "prefill"):
            module.prefill = prefill


def get_model_placement_stats(model: nn.Module) -> ModelPlacementStats:
    """placement.py:84-96: bytes of parameters on host and on device."""
    host_bytes = 0
    device_bytes = 0
    for param in model.parameters():
        param_bytes = param.numel() * param.element_size()
        if param.device.type == "cpu":
            host_bytes += param_bytes
        else:
            device_bytes += param_bytes
    total_bytes = host_bytes + device_bytes
    actual_offload_ratio = host_bytes / total_bytes if total_bytes else 0.0
    return ModelPlacementStats(host_bytes, device_bytes, actual_offload_ratio)


def offload_ratio_for_budget(model: nn.Module, hbm_budget_bytes: int, reserve_bytes: int = 0) -> float:
    """Fraction of the replaced linears' weight bytes that must live on the host
    so that everything else plus the rest of the linears fits in the budget.

    Bytes are counted at the 16-bit storage size the split keeps.  The result
    is clamped to [0, 1]; 0 means the model fits without offloading."""
    custom_types = _custom_linear_types()
    linear_bytes = 0
    other_bytes = 0
    custom_params = set()
    for m in model.modules():
        if isinstance(m, custom_types):
            for p in m.parameters(recurse=False):
                custom_params.add(id(p))
                if p is getattr(m, "bias", None):
                    other_bytes += p.numel() * 2
                else:
                    linear_bytes += p.numel() * 2
    for p in model.parameters():
        if id(p) not in custom_params:
            other_bytes += p.numel() * p.element_size()
    for b in model.buffers():
        other_bytes += b.numel() * b.element_size()
    if linear_bytes == 0:
        return 0.0
    room = hbm_budget_bytes - reserve_bytes - other_bytes
    return float(min(1.0, max(0.0, 1.0 - room / linear_bytes)))


def _place_horizontal_linear(name, module, offload_ratio, *, gpu_name, use_config, horizontal_config,
                             default_horizontal_config, allow_edges=False, host_side="first") -> None:
    """placement.py:99-130."""
    if not allow_edges and not 0.0 < offload_ratio < 1.0:
        raise ValueError(f"{name} is a horizontal Linear, so offload_ratio must be between 0 and 1; got {offload_ratio}")
    h_m, d_m, h_blocks, d_blocks, h_sms_per_row, d_sms_per_row = _resolve_horizontal_split_config(
        module, offload_ratio, gpu_name=gpu_name, use_config=use_config, horizontal_config=horizontal_config,
        default_horizontal_config=default_horizontal_config,
    )
    if allow_edges and h_m == 0 and d_m == 0:
        from .utils import split_horizontal

        h_m, d_m = split_horizontal((module.out_features, module.in_features), offload_ratio)
        if h_m == 0:
            d_m = module.out_features
    module.horizontal_split_weight(offload_ratio, h_blocks + d_blocks, h_blocks, h_sms_per_row, d_sms_per_row, h_m,
                                   d_m, host_side=host_side)


def _resolve_horizontal_split_config(module, offload_ratio, *, gpu_name, use_config, horizontal_config,
                                     default_horizontal_config):
    """placement.py:133-160, with B200 added to the built-in defaults."""
    if default_horizontal_config is not None and gpu_name in default_horizontal_config:
        config = default_horizontal_config[gpu_name]
    elif gpu_name == "GH200":
        config = (0, 0, 16, 112, 1, 1)
    elif gpu_name == "RTX6000":
        config = (0, 0, 8, 180, 1, 1)
    elif gpu_name == "B200":
        config = B200_DEFAULT_SPLIT
    else:
        raise NotImplementedError(f"GPU {gpu_name} not supported for horizontal split config")
    if not use_config:
        return config
    weight_shape = tuple(module.weight.shape)
    gpu_config = horizontal_config.get(gpu_name)
    if gpu_config is None:
        raise KeyError(f"Horizontal config for GPU {gpu_name} not found")
    if weight_shape not in gpu_config:
        raise KeyError(f"Weight shape {weight_shape} not found in horizontal config for {gpu_name}")
    return gpu_config[weight_shape]


def _move_non_custom_direct_tensors(module, custom_types, device) -> None:
    """placement.py:163-172."""
    if isinstance(module, custom_types):
        return
    _move_direct_parameters_and_buffers(module, device)
    for child in module.children():
        _move_non_custom_direct_tensors(child, custom_types, device)


def _move_direct_parameters_and_buffers(module: nn.Module, device) -> None:
    """placement.py:175-187."""
    with torch.no_grad():
        for param in module._parameters.values():
            if param is not None:
                param.data = param.data.to(device, non_blocking=True)
                if param.grad is not None:
                    param.grad.data = param.grad.data.to(device, non_blocking=True)
        for name, buffer in module._buffers.items():
            if buffer is not None:
                module._buffers[name] = buffer.to(device, non_blocking=True)


def _move_custom_linear_bias(module: nn.Module, device) -> None:
    """placement.py:190-197."""
    bias = getattr(module, "bias", None)
    if bias is None:
        return
    with torch.no_grad():
        bias.data = bias.data.to(device, non_blocking=True)
        if bias.grad is not None:
            bias.grad.data = bias.grad.data.to(device, non_blocking=True)


def _custom_linear_types() -> tuple[type[nn.Module], ...]:
    from .layers import Linear, LinearHorizontal, LinearHorizontalMulticast, LinearMulticast

    return (Linear, LinearHorizontal, LinearMulticast, LinearHorizontalMulticast)


def _is_horizontal_linear(module: Any) -> bool:
    return hasattr(module, "horizontal_split_weight")


def _is_host_linear(module: Any) -> bool:
    return hasattr(module, "move_weight_to_device")
