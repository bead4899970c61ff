"""Linear replacement entry point, keeping the interface of the reference's
app/python/linear_replacement.py:1-269.

The public surface is the reference's: ``LinearType``, the
``LinearReplacementConfig`` dataclass (same fields and defaults), the
``{set,get}_{opt,llama}_linear_config`` pair that stores a configuration on a
Hugging Face config as ``{opt,llama}_linear_*`` attributes,
``make_replacement_linear``, ``replace_{opt,llama}_linears`` and
``load_replaced_{opt,llama}_for_causal_lm``.

The implementation is table driven.  ``_STORED_FIELDS`` is a codec between
the dataclass and the config attributes (which fields are stored, their
defaults when absent, and how torch dtypes and devices are written as
strings).  ``_Family`` records (``_OPT``, ``_LLAMA``) describe, per model family, where each target linear
lives (decoder layer, attention block, MLP block, or the model itself), so one
routine swaps linears for every family.
"""
from __future__ import annotations

import dataclasses
from collections.abc import Callable, Iterable
from dataclasses import dataclass
from typing import Any, Literal

import torch
from torch import nn

LinearType = Literal["vanila", "host", "horizontal", "multicast", "horizontal_multicast"]

OPT_TARGET_LINEARS = ("q_proj", "k_proj", "v_proj", "out_proj", "fc1", "fc2")
OPT_PROJECTION_LINEARS = ("project_in", "project_out")
LLAMA_ATTENTION_LINEARS = ("q_proj", "k_proj", "v_proj", "o_proj")
LLAMA_MLP_LINEARS = ("gate_proj", "up_proj", "down_proj")
LLAMA_HEAD_LINEARS = ("lm_head",)
LLAMA_TARGET_LINEARS = LLAMA_ATTENTION_LINEARS + LLAMA_MLP_LINEARS + LLAMA_HEAD_LINEARS


@dataclass(frozen=True)
class LinearReplacementConfig:
    """Field names and defaults of linear_replacement.py:21-31."""

    linear_type: LinearType
    smem_size: int | None = None
    num_copy_blocks: int = 128
    device: torch.device | str | None = None
    dtype: torch.dtype | None = torch.float16
    multicast_kernel: bool | None = None
    include_embedding_projections: bool = False
    drop_bias: bool = True
    skip_init: bool = True


# ------------------------------------------------------------------ codec
def _dtype_name(dtype: torch.dtype | None) -> str | None:
    return None if dtype is None else str(dtype).rsplit(".", 1)[-1]


def _dtype_from_name(value: Any) -> torch.dtype | None:
    if value is None or isinstance(value, torch.dtype):
        return value
    return getattr(torch, str(value).rsplit(".", 1)[-1])


def _keep(value: Any) -> Any:
    return value


# Stored fields: (dataclass field, attribute suffix after "<family>_linear_",
# value when the attribute is absent, encode for the config, decode from it).
# include_embedding_projections is a call-time option and is not stored, as
# in linear_replacement.py:42-75.
_STORED_FIELDS: tuple[tuple[str, str, Any, Callable, Callable], ...] = (
    ("linear_type", "type", "vanila", _keep, _keep),
    ("smem_size", "smem_size", None, _keep, _keep),
    ("num_copy_blocks", "num_copy_blocks", 128, _keep, _keep),
    ("device", "device", None, lambda d: None if d is None else str(d), _keep),
    ("dtype", "dtype", "float16", _dtype_name, _dtype_from_name),
    ("multicast_kernel", "multicast_kernel", None, _keep, _keep),
    ("drop_bias", "drop_bias", True, _keep, _keep),
    ("skip_init", "skip_init", True, _keep, _keep),
)


def _coerce(replacement) -> LinearReplacementConfig:
    """A LinearReplacementConfig, or a bare linear type that stands for one."""
    if isinstance(replacement, LinearReplacementConfig):
        return replacement
    return LinearReplacementConfig(replacement)


def _store(config, family: str, replacement):
    cfg = _coerce(replacement)
    for field, attr, _, encode, _ in _STORED_FIELDS:
        setattr(config, f"{family}_linear_{attr}", encode(getattr(cfg, field)))
    return config


def _load(config, family: str) -> LinearReplacementConfig:
    values = {field: decode(getattr(config, f"{family}_linear_{attr}", absent))
              for field, attr, absent, _, decode in _STORED_FIELDS}
    return LinearReplacementConfig(**values)


def set_opt_linear_config(config, replacement):
    return _store(config, "opt", replacement)


def set_llama_linear_config(config, replacement):
    return _store(config, "llama", replacement)


def get_opt_linear_config(config) -> LinearReplacementConfig:
    return _load(config, "opt")


def get_llama_linear_config(config) -> LinearReplacementConfig:
    return _load(config, "llama")


# ------------------------------------------------------------- the modules
_MULTICAST_TYPES = frozenset({"multicast", "horizontal_multicast"})


def _module_class(linear_type: str):
    """The module class a linear type names (linear_replacement.py:88-107)."""
    if linear_type == "vanila":
        return nn.Linear
    from . import layers

    cls = {"host": "Linear", "horizontal": "LinearHorizontal", "multicast": "LinearMulticast",
           "horizontal_multicast": "LinearHorizontalMulticast"}.get(linear_type)
    if cls is None:
        raise ValueError(f"Unsupported linear type: {linear_type}")
    return getattr(layers, cls)


def _linear_kwargs(config: LinearReplacementConfig, bias: bool) -> dict:
    """Constructor arguments of the module for ``config`` (linear_replacement.py:
    110-131): a plain nn.Linear keeps its bias; the offloaded modules drop it
    unless asked not to, and take the shared-memory size of their kernel family
    (the multicast family unless ``multicast_kernel`` says otherwise)."""
    common = {"device": config.device, "dtype": config.dtype}
    if config.linear_type == "vanila":
        return {"bias": bias, **common}
    smem = config.smem_size
    if smem is None:
        from .utils import get_smem_size

        multicast = config.multicast_kernel
        smem = get_smem_size(multicast=config.linear_type in _MULTICAST_TYPES if multicast is None else multicast)
    return {"smem_size": smem, "num_copy_blocks": config.num_copy_blocks,
            "bias": bool(bias) and not config.drop_bias, **common, "skip_init": config.skip_init}


def make_replacement_linear(in_features: int, out_features: int, bias: bool, config: LinearReplacementConfig) -> nn.Module:
    """linear_replacement.py:78-85."""
    return _module_class(config.linear_type)(in_features, out_features, **_linear_kwargs(config, bias))


def _swap_in(old: nn.Linear, config: LinearReplacementConfig) -> nn.Module:
    """A replacement module holding ``old``'s weights (and bias, when kept); an
    unset device or dtype follows the old module (linear_replacement.py:152-177)."""
    w = old.weight
    config = dataclasses.replace(config, device=config.device or w.device, dtype=config.dtype or w.dtype)
    new = make_replacement_linear(old.in_features, old.out_features, old.bias is not None, config)
    with torch.no_grad():
        for name in ("weight", "bias"):
            dst, src = getattr(new, name, None), getattr(old, name, None)
            if dst is not None and src is not None:
                dst.copy_(src.to(device=dst.device, dtype=dst.dtype))
    return new


# ------------------------------------------------------- model families
@dataclass(frozen=True)
class _Family:
    """Where a model family keeps its replaceable linears.  ``layers`` yields the
    decoder layers; ``owner`` maps a per-layer linear's name to the attribute
    path of its parent inside a layer ("" = the layer itself), and other names
    are looked up under ``default_owner``; ``model_level`` maps names of
    linears outside the layers to (path of their parent, whether the parent
    must have the attribute)."""

    layers: Callable[[nn.Module], Iterable[nn.Module]]
    owner: dict[str, str]
    default_owner: str
    model_level: dict[str, tuple[str, bool]]


_OPT = _Family(
    layers=lambda m: m.model.decoder.layers,
    owner={n: "self_attn" for n in ("q_proj", "k_proj", "v_proj", "out_proj")},
    default_owner="",
    model_level={n: ("model.decoder", True) for n in OPT_PROJECTION_LINEARS},
)
_LLAMA = _Family(
    layers=lambda m: m.model.layers,
    owner={n: "self_attn" for n in LLAMA_ATTENTION_LINEARS},
    default_owner="mlp",
    model_level={"lm_head": ("", False)},
)


def _resolve(root: nn.Module, path: str) -> nn.Module:
    for part in filter(None, path.split(".")):
        root = getattr(root, part)
    return root


def _replace_at(parent: nn.Module, name: str, config: LinearReplacementConfig, required: bool = True) -> None:
    """Swaps ``parent.<name>``; a missing attribute raises AttributeError when
    ``required``, and an attribute set to None is left alone."""
    old = getattr(parent, name) if required else getattr(parent, name, None)
    if old is not None:
        setattr(parent, name, _swap_in(old, config))


def _replace(model: nn.Module, family: _Family, config: LinearReplacementConfig, targets: set[str]) -> nn.Module:
    per_layer = [n for n in targets if n not in family.model_level]
    for layer in family.layers(model):
        for name in per_layer:
            _replace_at(_resolve(layer, family.owner.get(name, family.default_owner)), name, config)
    for name, (path, required) in family.model_level.items():
        if name in targets:
            _replace_at(_resolve(model, path), name, config, required)
    return model


def replace_opt_linears(model: nn.Module, linear_type, target_names: Iterable[str] = OPT_TARGET_LINEARS) -> nn.Module:
    """OPT decoder q/k/v/out_proj and fc1/fc2, plus the embedding projections
    when the config includes them (linear_replacement.py:180-207)."""
    config = _coerce(linear_type)
    targets = set(target_names)
    if config.include_embedding_projections:
        targets |= set(OPT_PROJECTION_LINEARS)
    else:
        targets -= set(OPT_PROJECTION_LINEARS)
    return _replace(model, _OPT, config, targets)


def replace_llama_linears(model: nn.Module, linear_type, target_names: Iterable[str] = LLAMA_TARGET_LINEARS) -> nn.Module:
    """LLaMA attention and MLP linears and lm_head (linear_replacement.py:210-233)."""
    return _replace(model, _LLAMA, _coerce(linear_type), set(target_names))


def _load_replaced(model_cls_name: str, family: str, replace, path, linear_type, *args, **kwargs):
    import transformers

    if kwargs.get("config") is None:
        kwargs["config"] = transformers.AutoConfig.from_pretrained(path)
    _store(kwargs["config"], family, linear_type)
    model = getattr(transformers, model_cls_name).from_pretrained(path, *args, **kwargs)
    return replace(model, linear_type)


def load_replaced_opt_for_causal_lm(pretrained_model_name_or_path, linear_type, *args, **kwargs):
    """linear_replacement.py:236-251, on the stock transformers OPT model followed by
    ``replace_opt_linears`` (the reference builds its vendored OPT copy instead)."""
    return _load_replaced("OPTForCausalLM", "opt", replace_opt_linears, pretrained_model_name_or_path, linear_type,
                          *args, **kwargs)


def load_replaced_llama_for_causal_lm(pretrained_model_name_or_path, linear_type, *args, **kwargs):
    """linear_replacement.py:254-269 (stock transformers Llama + ``replace_llama_linears``)."""
    return _load_replaced("LlamaForCausalLM", "llama", replace_llama_linears, pretrained_model_name_or_path,
                          linear_type, *args, **kwargs)
