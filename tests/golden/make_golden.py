"""Generates the golden fixtures of tests/golden/ from the reference's own code.

Runs shouxulin/DirectAccessKernel's Python (app/python/*, opt_attention/*) on
CPU, in a container that has the reference checked out:

    python tests/golden/make_golden.py --ref /path/to/DirectAccessKernel

The reference's compiled `offload.runtime` (sm_90a/sm_120a only) is replaced by
a stub that records the arguments of build_tma_desc; CUDA tensors the reference
allocates are redirected to the CPU and pinned allocations to plain CPU memory.
Nothing here runs a reference GPU kernel.  What is pinned:

  split_horizontal.json  app/python/utils.py:18-45 over the configs' shapes/ratios
  tma_desc_args.json     app/python/utils.py:48-145 descriptor arguments
  linear_split.npz       LinearHorizontal.horizontal_split_weight slabs (checksums)
                         (app/python/layers/linearLayer.py:207-246)
  placement.json         place_model statistics and per-layer splits
                         (app/python/placement.py:35-160), replacement configs
                         (app/python/linear_replacement.py:21-75)
  linear_ref.npz         nn.Linear in FP32 (benchmark/benchmark_linear.py:121-123)
  attention_ref.npz      the attention hook's outputs (interface.py:142-189 ->
                         its transformers eager path) and vanila_llama's GQA
                         eager_attention_forward (vanila_llama.py:212-246)
  kv_cache.npz           PinnedStaticCache (app/python/pinned_static_cache.py)
                         after a prefill, single-token decode updates and a
                         scattered multi-token update

Inputs come from numpy's PCG64 generator with fixed seeds; the fixtures keep a
checksum of every input so tests can tell if a numpy version draws differently.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def checksum(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def gen(seed: int, shape, dtype=np.float16, scale: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(dtype)


def install_reference(ref: Path):
    repo = HERE.parent.parent
    sys.path[:] = [p for p in sys.path if Path(p or ".").resolve() != repo]
    for name in list(sys.modules):
        if name.split(".")[0] in ("app", "offload", "opt_attention", "split_attention"):
            del sys.modules[name]
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "opt_attention"))  # the inner opt_attention package
    import torch

    stub = types.ModuleType("offload")
    rt = types.ModuleType("offload.runtime")
    rt.NUM_SMS, rt.MAX_COPY_SMS, rt.BUFFER_SLOTS, rt.TILE_N = 132, 128, 3, 8
    rt.calls = []

    def build_tma_desc(base, shape, strides, box, elem_strides, swizzle):
        rt.calls.append({"tensor_shape": list(base.shape), "tensor_stride": list(base.stride()),
                         "shape": list(shape), "strides_bytes": list(strides), "box_dim": list(box),
                         "elem_strides": list(elem_strides), "swizzle": int(swizzle)})
        return torch.zeros(128, dtype=torch.uint8)

    rt.build_tma_desc = build_tma_desc
    rt.tensormap_replace_address = lambda desc, t: None
    rt.set_smem_size = lambda s, opcode=0: s
    stub.runtime = rt
    sys.modules["offload"] = stub
    sys.modules["offload.runtime"] = rt
    return rt


class redirect_cuda:
    """Sends torch.empty/zeros(device='cuda') to `target` and drops pin_memory."""

    def __init__(self, target: str):
        self.target = target

    def __enter__(self):
        import torch

        self.orig = {n: getattr(torch, n) for n in ("empty", "zeros")}

        def wrap(fn):
            def inner(*a, **k):
                if str(k.get("device", "")).startswith("cuda"):
                    k["device"] = self.target
                k.pop("pin_memory", None)
                return fn(*a, **k)

            return inner

        for n, f in self.orig.items():
            setattr(torch, n, wrap(f))
        return self

    def __exit__(self, *exc):
        import torch

        for n, f in self.orig.items():
            setattr(torch, n, f)


LLAMA8B_SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}
RATIOS = [0.0, 0.25, 0.5, 0.75, 1.0]


def make_split_tables(out: Path):
    from app.python import utils

    rows = []
    for name, (n, k) in {"config1": (4096, 4096), **LLAMA8B_SHAPES}.items():
        for r in RATIOS + [0.01, 0.03, 0.08, 0.33]:
            h, d = utils.split_horizontal((n, k), r)
            rows.append({"name": name, "shape": [n, k], "ratio": r, "h_m": h, "d_m": d})
    (out / "split_horizontal.json").write_text(json.dumps(rows, indent=1))


def make_desc_args(out: Path, rt):
    import torch
    from app.python import utils

    rt.calls.clear()
    cases = []
    for (k, m) in [(4096, 2048), (256, 192), (4096, 4096)]:
        w = torch.zeros(k, m, dtype=torch.float16)
        utils.build_tma_wgmma_mn(w, 64, 256)
        cases.append(("mn", [k, m], 64, 256, False))
        utils.build_tma_wgmma_mn(w, 64, 64, debug=True)
        cases.append(("mn", [k, m], 64, 64, True))
    for (n, k) in [(1, 4096), (8, 256), (16, 4096)]:
        x = torch.zeros(n, k, dtype=torch.float16)
        utils.build_tma_wgmma_k(x, 256, 8)
        cases.append(("k", [n, k], 256, 8, False))
        utils.build_tma_wgmma_k(x, 64, 256)
        cases.append(("k", [n, k], 64, 256, False))
    y = torch.zeros(3, 1, 4096, dtype=torch.float16)
    utils.build_tma_wgmma_mn(y.view(-1, 4096), 64, 8)
    cases.append(("mn", [3, 4096], 64, 8, False))
    rows = [{"kind": c[0], "matrix": c[1], "tile0": c[2], "tile1": c[3], "debug": c[4], **call}
            for c, call in zip(cases, rt.calls)]
    rows.append({"get_smem_size": utils.get_smem_size(False), "get_smem_size_multicast": utils.get_smem_size(True)})
    (out / "tma_desc_args.json").write_text(json.dumps(rows, indent=1))


def make_linear_split(out: Path):
    import torch
    from app.python.layers.linearLayer import LinearHorizontal

    w = gen(11, (256, 192), scale=0.02)
    res = {"w_seed": np.array(11), "w_sha": np.array(checksum(w))}
    for tag, (offload, h_m, d_m) in {"ratio": (0.5, 0, 0), "explicit": (0.0, 64, 192)}.items():
        with redirect_cuda("cpu"):
            lin = LinearHorizontal(192, 256, smem_size=0, num_copy_blocks=8, device="cpu", dtype=torch.float16,
                                   skip_init=True)
            lin.weight.data.copy_(torch.from_numpy(w))
            lin.horizontal_split_weight(offload, 8, 2, 1, 1, h_m, d_m)
        for part in ("weight_h", "weight_d"):
            t = getattr(lin, part).detach()
            res[f"{tag}_{part}_shape"] = np.array(list(t.shape))
            res[f"{tag}_{part}_stride"] = np.array(list(t.stride()))
            res[f"{tag}_{part}_sha"] = np.array(checksum(t.numpy()))
        res[f"{tag}_hd"] = np.array([lin.out_features_h, lin.out_features_d])
    np.savez_compressed(out / "linear_split.npz", **res)


def tiny_opt(seed: int):
    import torch
    from transformers import OPTConfig, OPTForCausalLM

    torch.manual_seed(seed)
    cfg = OPTConfig(hidden_size=128, num_attention_heads=2, ffn_dim=256, num_hidden_layers=2, vocab_size=96,
                    max_position_embeddings=64, word_embed_proj_dim=128)
    return OPTForCausalLM(cfg).to(torch.float16).eval()


def _placement_bytes(model):
    """Host/device bytes as get_model_placement_stats (placement.py:84-96) counts
    them on a GPU machine: the pinned slabs (weight_h, or the whole weight of a
    "host" Linear moved to "cpu") are host bytes, everything else device bytes."""
    host = 0
    total = 0
    for m in model.modules():
        for name, p in m.named_parameters(recurse=False):
            nbytes = p.numel() * p.element_size()
            total += nbytes
            if name == "weight_h" or getattr(m, "_golden_on_host", False) and name == "weight":
                host += nbytes
    return host, total - host


def make_placement(out: Path):
    import torch
    from app.python import linear_replacement as lr
    from app.python import placement

    res = {}
    for ratio in (0.25, 0.5, 0.75):
        model = tiny_opt(3)
        cfg = lr.LinearReplacementConfig("horizontal", device="cpu", dtype=torch.float16)
        lr.replace_opt_linears(model, cfg)
        with redirect_cuda("cpu"):
            placement.place_model(model, ratio, gpu_name="GH200", device="cpu", build_tma_desc=False)
        layers = {n: [m.out_features_h, m.out_features_d, m.num_copy_blocks, m.num_copy_blocks_host]
                  for n, m in model.named_modules() if hasattr(m, "out_features_h")}
        host, dev = _placement_bytes(model)
        res[str(ratio)] = {"host_bytes": host, "device_bytes": dev, "ratio": host / (host + dev), "layers": layers}
    # Whole weights on host ("host" type at ratio 1.0) or in HBM (ratio 0.3).
    for ratio in (1.0, 0.3):
        model = tiny_opt(4)
        lr.replace_opt_linears(model, lr.LinearReplacementConfig("host", device="cpu", dtype=torch.float16))
        with redirect_cuda("cpu"):
            placement.place_model(model, ratio, gpu_name="GH200", device="cpu", build_tma_desc=False)
        for m in model.modules():
            if hasattr(m, "move_weight_to_device"):
                m._golden_on_host = ratio >= 1.0
        host, dev = _placement_bytes(model)
        res[f"host_type_{ratio}"] = {"host_bytes": host, "device_bytes": dev, "ratio": host / (host + dev),
                                     "weight_shape": list(model.model.decoder.layers[0].fc1.weight.shape)}
    errors = {}
    for bad in (0.0, 1.0):
        model = tiny_opt(5)
        lr.replace_opt_linears(model, lr.LinearReplacementConfig("horizontal", device="cpu"))
        try:
            with redirect_cuda("cpu"):
                placement.place_model(model, bad, gpu_name="GH200", device="cpu", build_tma_desc=False)
        except Exception as e:  # noqa: BLE001
            errors[str(bad)] = type(e).__name__
    model = tiny_opt(6)
    lr.replace_opt_linears(model, lr.LinearReplacementConfig("horizontal", device="cpu"))
    try:
        with redirect_cuda("cpu"):
            placement.place_model(model, 0.5, gpu_name="A100", device="cpu", build_tma_desc=False)
    except Exception as e:  # noqa: BLE001
        errors["A100"] = type(e).__name__
    model = tiny_opt(7)
    lr.replace_opt_linears(model, lr.LinearReplacementConfig("horizontal", device="cpu"))
    try:
        with redirect_cuda("cpu"):
            placement.place_model(model, 0.5, gpu_name="RTX6000", use_config=True, device="cpu")
    except Exception as e:  # noqa: BLE001
        errors["missing_shape"] = type(e).__name__
    res["errors"] = errors
    res["tables"] = {g: {f"{k[0]}x{k[1]}": list(v) for k, v in t.items()}
                     for g, t in placement.DEFAULT_HORIZONTAL_CONFIG.items()}
    conf = types.SimpleNamespace()
    lr.set_opt_linear_config(conf, lr.LinearReplacementConfig("horizontal_multicast", num_copy_blocks=64,
                                                              dtype=torch.bfloat16, drop_bias=False))
    res["opt_config_attrs"] = dict(vars(conf))
    got = lr.get_opt_linear_config(conf)
    res["opt_config_roundtrip"] = {"linear_type": got.linear_type, "num_copy_blocks": got.num_copy_blocks,
                                   "dtype": str(got.dtype), "drop_bias": got.drop_bias}
    res["kwargs_horizontal"] = {k: v if isinstance(v, (int, bool, type(None))) else str(v)
                                for k, v in lr._linear_kwargs(lr.LinearReplacementConfig("horizontal"), True).items()}
    res["kwargs_multicast"] = {k: v if isinstance(v, (int, bool, type(None))) else str(v)
                               for k, v in lr._linear_kwargs(lr.LinearReplacementConfig("multicast"), False).items()}
    (out / "placement.json").write_text(json.dumps(res, indent=1, default=str))


def make_linear_ref(out: Path):
    import torch

    res = {}
    for i, (ntok, n, k) in enumerate([(1, 128, 512), (3, 192, 256), (8, 256, 320), (17, 128, 256)]):
        x = gen(100 + i, (ntok, k))
        w = gen(200 + i, (n, k), scale=0.02)
        lin = torch.nn.Linear(k, n, bias=False)
        with torch.no_grad():
            lin.weight.copy_(torch.from_numpy(w.astype(np.float32)))
            y = lin(torch.from_numpy(x.astype(np.float32))).numpy()
        res[f"case{i}_shape"] = np.array([ntok, n, k])
        res[f"case{i}_seeds"] = np.array([100 + i, 200 + i])
        res[f"case{i}_y"] = y
        res[f"case{i}_x_sha"] = np.array(checksum(x))
        res[f"case{i}_w_sha"] = np.array(checksum(w))
    np.savez_compressed(out / "linear_ref.npz", **res)


def make_attention_ref(out: Path):
    import torch
    from opt_attention.interface import opt_attention_forward

    module = torch.nn.Module().eval()
    res = {}
    cases = [
        # name, B, H, S, host_size, dtype, mask
        ("mha_split", 4, 2, 128, 2, np.float32, False),
        ("mha_mask", 3, 2, 192, 1, np.float32, True),
        ("all_host", 2, 2, 64, 2, np.float32, False),
        ("all_gpu", 2, 2, 64, 0, np.float32, False),
        ("mha_fp16", 2, 2, 128, 1, np.float16, False),
    ]
    for ci, (name, B, H, S, host, dt, use_mask) in enumerate(cases):
        seeds = [300 + 10 * ci + j for j in range(4)]
        q = gen(seeds[0], (B, H, 1, 128)) / np.float16(math.sqrt(128))
        k = gen(seeds[1], (B, H, S, 128))
        v = gen(seeds[2], (B, H, S, 128))
        mask = None
        if use_mask:
            keep = np.random.default_rng(seeds[3]).integers(S // 2, S + 1, size=B)
            mask = np.zeros((B, 1, 1, S), np.float32)
            for b in range(B):
                mask[b, :, :, keep[b]:] = np.finfo(np.float32).min
        t = lambda a: torch.from_numpy(a.astype(dt))  # noqa: E731
        kt, vt = t(k), t(v)
        got, _ = opt_attention_forward(module, t(q), kt[host:], vt[host:],
                                       torch.from_numpy(mask) if mask is not None else None, dropout=0.0,
                                       scaling=1.0 / math.sqrt(128), key_host=kt[:host], value_host=vt[:host],
                                       host_size=host)
        res[f"{name}_cfg"] = np.array([B, H, S, host, 1 if dt == np.float16 else 0, 1 if use_mask else 0])
        res[f"{name}_seeds"] = np.array(seeds)
        res[f"{name}_out"] = got.float().numpy()
        res[f"{name}_sha"] = np.array(checksum(np.concatenate([q.ravel(), k.ravel(), v.ravel()])))
        if mask is not None:
            res[f"{name}_mask"] = mask
    # GQA through the reference's Llama eager attention (repeat_kv).
    from app.python.llama.vanila_llama import eager_attention_forward as llama_eager

    mod = torch.nn.Module().eval()
    mod.num_key_value_groups = 4
    B, Hq, Hkv, S = 2, 8, 2, 96
    seeds = [400, 401, 402]
    q = gen(seeds[0], (B, Hq, 1, 128)) / np.float16(math.sqrt(128))
    k = gen(seeds[1], (B, Hkv, S, 128))
    v = gen(seeds[2], (B, Hkv, S, 128))
    got, _ = llama_eager(mod, torch.from_numpy(q.astype(np.float32)), torch.from_numpy(k.astype(np.float32)),
                         torch.from_numpy(v.astype(np.float32)), None, scaling=1.0 / math.sqrt(128), dropout=0.0)
    res["gqa_cfg"] = np.array([B, Hq, Hkv, S])
    res["gqa_seeds"] = np.array(seeds)
    res["gqa_out"] = got.float().numpy()
    res["gqa_sha"] = np.array(checksum(np.concatenate([q.ravel(), k.ravel(), v.ravel()])))
    np.savez_compressed(out / "attention_ref.npz", **res)


# The host-KV cache update sequence: (cache_position or None, seed) per update,
# applied to both layers (layer 1 always with explicit positions).
KV_CACHE = {"layers": 2, "batch": 3, "hidden": 64, "heads": 4, "kv_heads": 2, "max_len": 48}
KV_UPDATES = [(None, 500)] + [([t], 501 + t) for t in range(20, 30)] + [([35, 31, 33], 540)]
KV_PREFILL = 20


def kv_update_positions(i: int):
    pos, _ = KV_UPDATES[i]
    return list(range(KV_PREFILL)) if pos is None else pos


def make_kv_cache(out: Path):
    import torch
    from app.python.pinned_static_cache import PinnedStaticCache

    c = KV_CACHE
    cfg = types.SimpleNamespace(num_hidden_layers=c["layers"], hidden_size=c["hidden"],
                                num_attention_heads=c["heads"], num_key_value_heads=c["kv_heads"])
    d = c["hidden"] // c["heads"]
    with redirect_cuda("cpu"):
        cache = PinnedStaticCache(cfg, c["batch"], c["max_len"], torch.float16)
    shas = []
    for i, (pos, seed) in enumerate(KV_UPDATES):
        T = len(kv_update_positions(i))
        k = gen(seed, (c["batch"], c["kv_heads"], T, d))
        v = gen(seed + 1000, (c["batch"], c["kv_heads"], T, d))
        shas.append(checksum(np.concatenate([k.ravel(), v.ravel()])))
        for layer in range(c["layers"]):
            kw = None
            if pos is not None or layer == 1:
                kw = {"cache_position": torch.tensor(kv_update_positions(i), dtype=torch.long)}
            cache.update(torch.from_numpy(k), torch.from_numpy(v), layer, kw)
    res = {"cfg": np.array([c[n] for n in ("layers", "batch", "hidden", "heads", "kv_heads", "max_len")]),
           "seq_lengths": np.array([cache.get_seq_length(layer) for layer in range(c["layers"])]),
           "input_sha": np.array(shas)}
    for layer in range(c["layers"]):
        res[f"k{layer}"] = cache.key_cache[layer].numpy()
        res[f"v{layer}"] = cache.value_cache[layer].numpy()
    np.savez_compressed(out / "kv_cache.npz", **res)


MAKERS = ["split_tables", "desc_args", "linear_split", "placement", "linear_ref", "attention_ref", "kv_cache"]


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ref", required=True, help="checkout of shouxulin/DirectAccessKernel")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", nargs="*", choices=MAKERS, help="regenerate only these fixtures")
    args = ap.parse_args()
    ref = Path(args.ref)
    if not (ref / "app" / "python" / "utils.py").exists():
        raise SystemExit(f"{ref} is not a DirectAccessKernel checkout")
    out = Path(args.out)
    rt = install_reference(ref)
    want = set(args.only or MAKERS)
    if "split_tables" in want:
        make_split_tables(out)
    if "desc_args" in want:
        make_desc_args(out, rt)
    if "linear_split" in want:
        make_linear_split(out)
    if "placement" in want:
        make_placement(out)
    if "linear_ref" in want:
        make_linear_ref(out)
    if "attention_ref" in want:
        make_attention_ref(out)
    if "kv_cache" in want:
        make_kv_cache(out)
    for p in sorted(out.glob("*.json")) + sorted(out.glob("*.npz")):
        print(f"{p.name:24s} {p.stat().st_size:8d} B")


if __name__ == "__main__":
    main()
