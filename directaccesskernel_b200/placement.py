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

# Split every horizontal module of a GPU gets when no per-shape table is used.
# The GH200 and RTX6000 rows are the reference's built-in values
# (placement.py:141-146); a caller's default_horizontal_config overrides them.
_BUILTIN_SPLIT = {"GH200": (0, 0, 16, 112, 1, 1), "RTX6000": (0, 0, 8, 180, 1, 1), "B200": B200_DEFAULT_SPLIT}


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
    h_m, d_m, h_blocks, d_blocks, h_sms_per_row, d_sms_per_row = _split_plan(
        module, gpu_name=gpu_name, use_config=use_config, horizontal_config=horizontal_config,
        default_horizontal_config=default_horizontal_config,
    )
    if allow_edges and h_m == 0 and d_m == 0:
        from .utils import split_horizontal

        h_m, d_m = split_horizontal((module.out_features, module.in_features), offload_ratio)
        if h_m == 0:
            d_m = module.out_features
    module.horizontal_split_weight(offload_ratio, h_blocks + d_blocks, h_blocks, h_sms_per_row, d_sms_per_row, h_m,
                                   d_m, host_side=host_side)


def _split_plan(module, *, gpu_name, use_config, horizontal_config, default_horizontal_config):
    """The split tuple of one horizontal module (placement.py:133-160): the
    GPU's default row, or with ``use_config`` the row of its weight shape in
    ``horizontal_config[gpu_name]``.  A GPU with no default row raises
    NotImplementedError, also when a shape table would be used; a missing table
    or shape raises KeyError."""
    defaults = dict(_BUILTIN_SPLIT)
    defaults.update(default_horizontal_config or {})
    if gpu_name not in defaults:
        raise NotImplementedError(f"GPU {gpu_name} not supported for horizontal split config")
    if not use_config:
        return defaults[gpu_name]
    table = horizontal_config.get(gpu_name)
    if table is None:
        raise KeyError(f"Horizontal config for GPU {gpu_name} not found")
    shape = tuple(module.weight.shape)
    if shape not in table:
        raise KeyError(f"Weight shape {shape} not found in horizontal config for {gpu_name}")
    return table[shape]


def _move_param(param, device) -> None:
    """Moves a parameter's data (and gradient) to ``device`` in place, keeping
    the Parameter object that modules and optimizers hold."""
    if param is None:
        return
    param.data = param.data.to(device, non_blocking=True)
    if param.grad is not None:
        param.grad.data = param.grad.data.to(device, non_blocking=True)


def _move_non_custom_direct_tensors(model: nn.Module, custom_types, device) -> None:
    """Every parameter and buffer of ``model`` outside the replaced linears goes
    to ``device`` (placement.py:163-187); the replaced linears' weights are
    placed by their splits.  Walks the module tree without recursion."""
    pending = [model]
    with torch.no_grad():
        while pending:
            module = pending.pop()
            if isinstance(module, custom_types):
                continue
            for param in module._parameters.values():
                _move_param(param, device)
            for key, buf in list(module._buffers.items()):
                if buf is not None:
                    module._buffers[key] = buf.to(device, non_blocking=True)
            pending.extend(module.children())


def _move_custom_linear_bias(module: nn.Module, device) -> None:
    """A replaced linear's bias lives with the rest of the model on ``device``
    (placement.py:190-197); its weight stays where the split put it."""
    with torch.no_grad():
        _move_param(getattr(module, "bias", None), device)


def _custom_linear_types() -> tuple[type[nn.Module], ...]:
    from .layers import Linear, LinearHorizontal, LinearHorizontalMulticast, LinearMulticast

    return (Linear, LinearHorizontal, LinearMulticast, LinearHorizontalMulticast)


def _is_horizontal_linear(module: Any) -> bool:
    return hasattr(module, "horizontal_split_weight")


def _is_host_linear(module: Any) -> bool:
    return hasattr(module, "move_weight_to_device")
