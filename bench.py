"""Benchmark of the direct-access offloading hot path on B200.

Default workload: the Llama-3-8B linear sweep - weights
qkv [6144x4096], o [4096x4096], gate_up [28672x4096], down [4096x14336], fp16
~ N(0, 0.02); activations M in {1, 4, 16, 64} tokens ~ N(0, 1); host offload
ratio r in {0, .25, .5, .75, 1}.  One step is one pass over the whole sweep
(80 linear layers, 8.7 GB of weight reads), each layer run through the
reference-facing module API (LinearHorizontal for 0 < r < 1, Linear on "cuda"
/ "cpu" for r = 0 / 1, as placement.py places them).  Weights total 436 MB
per (M, r) pass, larger than the 126 MB L2, so no flush is needed between
steps.  ``--workload attention`` runs BASELINE config 3 instead;
``--workload prefill`` runs the same layers at 512 tokens (the large-N path),
against a roofline that adds the tensor-core term 2 M N K / peak.

Metric: effective weight GB/s (weight bytes / time, benchmark_linear.py:341),
with a roofline of max((1-r) W / HBM, r W / host link) per layer.

Usage (driver contract): python bench.py [--gpus N] [--steps K] [--warmup W]
[--impl reference]; under torchrun one process per GPU.  The linear workloads
then run tensor-parallel (strong scaling): every layer is column-parallel, each
GPU streams its shard of the weights from its own HBM and over its own host
link, and NCCL all-gathers y after every layer.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

LLAMA8B = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}
# One tensor-parallel rank's layers of the Llama-3-70B decoder at TP 8 (config 5).
LLAMA70B_TP8 = {"qkv": (1280, 8192), "o": (8192, 1024), "gate_up": (7168, 8192), "down": (8192, 3584)}
TOKENS = (1, 4, 16, 64)
RATIOS = (0.0, 0.25, 0.5, 0.75, 1.0)
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TFLOPS = 1590.0
FALLBACK_TFLOPS_SUSTAINED = 1400.0
# Tokens per launch of the tcgen05 linear kernel; larger batches run in chunks.
MMA_MAX_TOKENS = 256
# Peer copy bandwidth per direction per GPU over NVLink 5 measured on this
# pool's B200 boxes (900 GB/s nominal): the roofline term of the all-gather.
NVLINK_GBS = 770.0
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch divided by
# the launch's device-tier bytes ((1 - r) W + x + y), measured with ncu on
# full-size launches of both linear kernels on the Llama-3-8B layers at r = 0
# and 0.5: 1.000-1.004, mean 1.002.  The host tier's bytes cross PCIe and never
# touch DRAM.
DRAM_PER_DEVICE_BYTE = 1.002
# Same for the decode-attention kernel on BASELINE config 3 (one full-size
# launch): 541.6 MB of DRAM traffic for 536.9 MB of device-resident K/V.
ATTN_DRAM_PER_DEVICE_BYTE = 1.0088


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["linear", "prefill", "attention", "opt66b", "llama70b", "plan-sweep",
                                           "read-ceiling"],
                    default="linear",
                    help="prefill: the Llama-3-8B layers at 512 tokens, r in {0, 0.5, 1} (large-N path)")
    ap.add_argument("--layers", type=int, default=80, help="llama70b: decoder layers")
    ap.add_argument("--batch", type=int, default=32, help="llama70b: sequences")
    ap.add_argument("--ctx", type=int, default=16384, help="llama70b: context tokens per sequence")
    ap.add_argument("--breakdown", action="store_true",
                    help="llama70b: after the timed region, one eager step with CUDA events around every op group "
                         "(per-op milliseconds in the JSON line)")
    ap.add_argument("--rank-of-tp", type=int, default=1,
                    help="llama70b on 1 GPU: build one rank of a TP-N decoder (heads, KV heads, FFN and vocabulary "
                         "divided by N) to profile its kernels on one GPU; there is no all-reduce")
    ap.add_argument("--nccl-allreduce", action="store_true",
                    help="llama70b: NCCL all-reduce after o and down (by default the decoder times the fused "
                         "reduction and NCCL at set-up and keeps the faster)")
    ap.add_argument("--no-balance", action="store_true",
                    help="llama70b: same host fraction on every rank (default: balanced by host bandwidth)")
    ap.add_argument("--host-fraction", type=float, default=None,
                    help="llama70b: fixed host fraction of weights and KV (default: from the HBM budget)")
    ap.add_argument("--hbm-budget-gb", type=float, default=None,
                    help="HBM budget in GB (opt66b: weights, default 96; llama70b: per GPU, default 60)")
    ap.add_argument("--prompt-len", type=int, default=512, help="opt66b: prompt tokens")
    ap.add_argument("--tokens", type=str, default=None, help="comma list overriding the M sweep")
    ap.add_argument("--ratios", type=str, default=None, help="comma list overriding the ratio sweep")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-row-parallel", action="store_true",
                    help="linear sweep under torchrun: skip the row-parallel all-reduce check")
    ap.add_argument("--details", type=str, default=None, help="write per-layer results (JSON) here")
    ap.add_argument("--sweep-shapes", choices=["llama8b", "llama70b-tp8"], default="llama8b",
                    help="plan-sweep: the Llama-3-8B layers, or one TP8 rank's Llama-3-70B layers")
    return ap.parse_args()


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_tflops(sustained: bool = False) -> tuple[float, str]:
    """Dense bf16/fp16 tensor throughput (cuBLAS GEMM) from MEASURED_PEAKS.json."""
    p = REPO / "MEASURED_PEAKS.json"
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    if p.exists():
        d = json.loads(p.read_text())
        if key in d:
            return float(d[key]), "measured"
    return (FALLBACK_TFLOPS_SUSTAINED if sustained else FALLBACK_TFLOPS), "fallback"


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"dak_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in self.path.read_text().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9 or not f[1].replace(".", "").isdigit():
                    continue
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
                for n, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        except OSError:
            pass
        finally:
            try:
                self.path.unlink()
            except OSError:
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ link probes
def host_link_probe(torch, runtime, world: int = 1):
    """Host->GPU read bandwidth: DMA copy of pinned memory and the TMA read probe.
    Under torchrun every rank measures at the same time (barriers between the
    phases), so the figures include the contention of all GPUs on the host."""
    def sync():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
            torch.cuda.synchronize()

    n = 1 << 30
    src = torch.empty(n, dtype=torch.uint8).pin_memory()
    src.fill_(1)
    dst = torch.empty(n, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        dst.copy_(src, non_blocking=True)
    sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        dst.copy_(src, non_blocking=True)
    e1.record()
    e1.synchronize()
    dma = 3 * n / (e0.elapsed_time(e1) * 1e-3) / 1e9
    best = 0.0
    for ctas in (16, 32, 64):
        runtime.probe_stream_read(src, ctas, 4, 32768)
        sync()
        e0.record()
        runtime.probe_stream_read(src, ctas, 4, 32768)
        e1.record()
        e1.synchronize()
        best = max(best, n / (e0.elapsed_time(e1) * 1e-3) / 1e9)
    del src, dst
    return dma, best


def hbm_read_probe(torch, runtime):
    n = 2 << 30
    src = torch.empty(n, dtype=torch.uint8, device="cuda")
    runtime.probe_stream_read(src, runtime.NUM_SMS * 2, 4, 16384)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    runtime.probe_stream_read(src, runtime.NUM_SMS * 2, 4, 16384)
    e1.record()
    e1.synchronize()
    return n / (e0.elapsed_time(e1) * 1e-3) / 1e9


# ---------------------------------------------------------------- workload
def layer_roofline(m: int, n: int, k: int, host_bytes: int, hbm_gbs: float, host_gbs: float,
                   tflops: float, dtype_bytes: int = 2) -> tuple[str, float]:
    """Lower bound (seconds) of one y[m, n] = x[m, k] W^T call whose weight has
    ``host_bytes`` on the host: the slowest of the HBM stream (device weight rows
    plus x and y), the host-link stream and the tensor-core work."""
    w_bytes = n * k * dtype_bytes
    io = (m * k + m * n) * dtype_bytes
    terms = {"hbm": (w_bytes - host_bytes + io) / (hbm_gbs * 1e9),
             "host": host_bytes / (host_gbs * 1e9),
             "tensor": 2.0 * m * n * k / (tflops * 1e12)}
    which = max(terms, key=terms.get)
    return which, terms[which]


def build_layers(torch, tokens, ratios, seed=0, rank=0, world=1, host_frac=None, keep_weights=False):
    """One module per (shape, ratio), placed as placement.py places it.

    With ``world`` > 1 every layer is column-parallel (tensor parallel): every
    rank generates the same full weight, keeps output features [rank N/G,
    (rank+1) N/G) as an offloaded module split between its own HBM and its own
    pinned host memory, and all-gathers y after each call.  ``host_frac[r]`` is
    this rank's host fraction for sweep ratio r (the mean over ranks is r)."""
    from directaccesskernel_b200.layers import Linear, LinearHorizontal
    from directaccesskernel_b200.utils import get_smem_size, split_horizontal

    g = torch.Generator(device="cuda").manual_seed(seed)
    layers, weights = [], {}
    for name, (n, k) in LLAMA8B.items():
        w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).half()
        if keep_weights:
            weights[name] = w.cpu()
        for r in ratios:
            if world > 1:
                from directaccesskernel_b200.tp import ColumnParallelLinear, make_offloaded_shard, shard_rows

                rr = host_frac[r] if host_frac else r
                local = make_offloaded_shard(shard_rows(w, rank, world), rr)
                if isinstance(local, LinearHorizontal):
                    host_rows = local.out_features_h
                else:
                    host_rows = n // world if local.weight.device.type == "cpu" else 0
                lin = ColumnParallelLinear(local, n)
                layers.append({"name": name, "n": n, "k": k, "ratio": r, "rank_ratio": rr, "mod": lin,
                               "w_bytes": n * k * 2, "rank_n": n // world, "host_bytes": host_rows * k * 2})
                continue
            if 0.0 < r < 1.0:
                lin = LinearHorizontal(k, n, get_smem_size(), 0, device="cuda", dtype=torch.float16, skip_init=True)
                with torch.no_grad():
                    lin.weight.copy_(w)
                h_m, d_m = split_horizontal((n, k), r)
                lin.horizontal_split_weight(r, 0, 0, 1, 1, h_m, d_m)
                lin.build_tma_desc()
                host_bytes = h_m * k * 2
            else:
                lin = Linear(k, n, get_smem_size(), 0, device="cuda", dtype=torch.float16, skip_init=True)
                with torch.no_grad():
                    lin.weight.copy_(w)
                lin.move_weight_to_device("cpu" if r >= 1.0 else "cuda")
                lin.build_tma_desc()
                host_bytes = n * k * 2 if r >= 1.0 else 0
            layers.append({"name": name, "n": n, "k": k, "ratio": r, "rank_ratio": r, "mod": lin, "w_bytes": n * k * 2,
                           "rank_n": n, "host_bytes": host_bytes})
        del w
    torch.cuda.synchronize()
    return (layers, weights) if keep_weights else layers


def linear_sweep(args):
    """(prefill, tokens, ratios) of the linear workloads."""
    prefill = args.workload == "prefill"
    tokens = [int(t) for t in args.tokens.split(",")] if args.tokens else ([512] if prefill else list(TOKENS))
    ratios = ([float(r) for r in args.ratios.split(",")] if args.ratios
              else ([0.0, 0.5, 1.0] if prefill else list(RATIOS)))
    return prefill, tokens, ratios


def linear_metric_config(prefill, tokens, ratios, world):
    """Metric name and `config` of the linear workloads, the same for both arms."""
    if prefill:
        metric = f"offloaded linear effective weight GB/s (Llama-3-8B layers, prefill M={tokens})"
        workload = (f"large-N prefill: Llama-3-8B qkv/o/gate_up/down x M{tokens} x r{ratios}; up to "
                    f"{2 * MMA_MAX_TOKENS} tokens per launch (HBM-only layers as grid rows of up to "
                    f"{MMA_MAX_TOKENS} tokens)")
    else:
        metric = "offloaded GEMV effective weight GB/s (Llama-3-8B linear sweep)"
        workload = "BASELINE config 2: Llama-3-8B qkv/o/gate_up/down x M{1,4,16,64} x r{0,.25,.5,.75,1}"
    calls = len(tokens) * len(ratios) * len(LLAMA8B)
    config = {"workload": workload,
              "tokens": tokens, "ratios": ratios, "layers_per_step": calls,
              "weight_bytes_per_step": len(tokens) * len(ratios) * sum(2 * n * k for (n, k) in LLAMA8B.values()),
              "host_rows": "first (reference split_horizontal)",
              "l2": "no flush: 436 MB of weights per (M, r) pass exceed the 126 MB L2",
              "timing": f"device: one CUDA graph per step ({calls} launches) replayed K times; "
                        "per-launch breakdown: per-layer graphs back to back with events between",
              "parallelism": "single GPU (tp1)"}
    if world > 1:
        config["parallelism"] = (f"tp{world}: every layer column-parallel (output features sharded over {world} "
                                 "GPUs, each shard split between its own HBM and its own pinned host memory), "
                                 "y all-gathered over NCCL after each layer; the whole job streams each weight once")
    return metric, config


def linear_parity(torch, layers, calls, outputs, weights, x_dev, tol=1e-2):
    """Max relative error (max|y - ref| / max|ref|) of every call's output against
    the reference's own CPU computation of the layer, torch F.linear in FP32 on
    the host cores (benchmark_linear.py:121-123: nn.Linear on float copies)."""
    import torch.nn.functional as F

    worst, refs = 0.0, {}
    for (l, m), y in zip(calls, outputs):
        key = (l["name"], m)
        if key not in refs:
            x = x_dev[(m, l["k"])].reshape(m, l["k"]).float().cpu()
            refs[key] = F.linear(x, weights[l["name"]].float())
        ref = refs[key]
        err = ((y.reshape(m, -1).float().cpu() - ref).abs().max() / ref.abs().max()).item()
        worst = max(worst, err)
    return {"max_rel_err": round(worst, 6), "cases": len(calls), "tolerance": tol, "ok": worst <= tol,
            "reference": "torch F.linear(x.float(), W.float()) on the host cores (benchmark_linear.py:121-123)",
            "checked": "rank 0, on the full (all-gathered) outputs of every layer call"}


def row_parallel_check(torch, rank, world, steps=10, tol=1e-2):
    """The row-parallel layers of a tensor-parallel decoder (o and down of the
    Llama-3-8B shapes), with input features sharded over the ranks and half of
    each rank's output features in its pinned host memory.  Every rank's
    partial y is summed over the ranks three ways: by the all-reduce fused into
    the linear kernel (``dak_linear_split_allreduce``), by the linear followed
    by an NCCL all-reduce, and, where NVSwitch multicast is available, by the
    consumer-side reduction the decoder uses (publish-only linear, then
    ``dak_rmsnorm_allreduce`` adds the sum to a residual and normalises).
    Rank 0 checks each against torch F.linear in FP32 on the host cores on the
    full weight, and every rank checks that its sum equals rank 0's.  Each way
    is then timed per call: a CUDA graph of ``steps`` calls, max over ranks."""
    import torch.distributed as dist
    import torch.nn.functional as F

    from directaccesskernel_b200 import runtime
    from directaccesskernel_b200.tp import SymmetricAllReduce

    shapes = {name: LLAMA8B[name] for name in ("o", "down")}
    ntoks = (1, 32)
    slot = max(ntoks) * max(n for n, _ in shapes.values())
    ar = SymmetricAllReduce(slot_elems=slot)
    arc = SymmetricAllReduce(slot_elems=slot, consumer_reduces=True)
    g = torch.Generator(device="cuda").manual_seed(4321)  # the same draws on every rank
    worst = {"fused_linear": 0.0, "linear_nccl": 0.0, "rmsnorm_residual": 0.0, "rmsnorm_out": 0.0,
             "ranks_differ": 0.0}
    calls = {}

    def rel(a, b):
        return ((a.float().cpu() - b.float()).abs().max() / b.float().abs().max()).item()

    def same_as_rank0(t):
        t0 = t.clone()
        dist.broadcast(t0, 0)
        return (t.float() - t0.float()).abs().max().item()

    for name, (n, k) in shapes.items():
        if k % world:
            raise RuntimeError(f"{name}: {k} input features do not split over {world} ranks")
        kr = k // world
        w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).half()
        wt = w[:, rank * kr:(rank + 1) * kr].t().contiguous()  # this rank's transposed shard [kr, n]
        w_host = wt[:, :n // 2].cpu().pin_memory()
        w_dev = wt[:, n // 2:].contiguous()
        wn = (1 + 0.1 * torch.randn(n, generator=g, device="cuda")).half()
        w_cpu = w.float().cpu() if rank == 0 else None
        del w
        for m in ntoks:
            x = torch.randn(m, k, generator=g, device="cuda").half()
            res = torch.randn(m, n, generator=g, device="cuda").half()
            xr = x[:, rank * kr:(rank + 1) * kr].contiguous()
            y = torch.empty(m, n, dtype=torch.float16, device="cuda")
            y2 = torch.empty_like(y)
            runtime.linear_split(xr, y, w_host, w_dev, allreduce=ar)
            runtime.linear_split(xr, y2, w_host, w_dev)
            dist.all_reduce(y2)
            state, out = res.clone(), torch.empty_like(res)
            if arc.publish_only:
                yc = torch.empty_like(y)  # layout only: a publish-only call leaves it unwritten
                runtime.linear_split(xr, yc, w_host, w_dev, allreduce=arc)
                arc.rmsnorm(yc, state, wn, 1e-5, out)
            torch.cuda.synchronize()
            worst["ranks_differ"] = max(worst["ranks_differ"], same_as_rank0(y), same_as_rank0(state))
            if rank == 0:
                ref = F.linear(x.float().cpu(), w_cpu)
                worst["fused_linear"] = max(worst["fused_linear"], rel(y, ref))
                worst["linear_nccl"] = max(worst["linear_nccl"], rel(y2, ref))
                if arc.publish_only:
                    h = ref.half() + res.cpu()
                    hf = h.float()
                    o_ref = wn.cpu() * (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5)).half()
                    worst["rmsnorm_residual"] = max(worst["rmsnorm_residual"], rel(state, h))
                    worst["rmsnorm_out"] = max(worst["rmsnorm_out"], rel(out, o_ref))
            # timed with the whole shard in HBM, so the reduction is not hidden
            # behind the host link
            calls[(name, m)] = (xr, y, y2, None, wt, state, out, wn)

    # ---- per-call device time of each way, at 32 tokens (a decode batch), with
    # each rank's shard all in HBM
    stream = torch.cuda.current_stream()
    ways = {"fused_linear": lambda c: runtime.linear_split(c[0], c[1], c[3], c[4], allreduce=ar),
            "linear_nccl": lambda c: (runtime.linear_split(c[0], c[2], c[3], c[4]), dist.all_reduce(c[2]))}
    if arc.publish_only:
        ways["consumer_rmsnorm"] = lambda c: (runtime.linear_split(c[0], c[1], c[3], c[4], allreduce=arc),
                                              arc.rmsnorm(c[1], c[5], c[7], 1e-5, c[6]))
    us = {}
    for way, fn in ways.items():
        for name in shapes:
            c = calls[(name, 32)]
            for _ in range(3):
                fn(c)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(steps):
                    fn(c)
            graph.replay()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            us[f"{way}/{name}"] = e0.elapsed_time(e1) * 1e3 / steps
            del graph  # graphs that hold NCCL calls go before the process group
    torch.cuda.synchronize()
    status = runtime.device_status()
    t = torch.tensor(list(us.values()) + [float(status != 0)], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = dict(zip(us, [round(v, 2) for v in t.tolist()[:-1]]))
    errs = torch.tensor(list(worst.values()), dtype=torch.float64, device="cuda")
    dist.all_reduce(errs, op=dist.ReduceOp.MAX)
    worst = dict(zip(worst, [round(v, 6) for v in errs.tolist()]))
    checked = ["fused_linear", "linear_nccl"] + (["rmsnorm_residual", "rmsnorm_out"] if arc.publish_only else [])
    return {"layers": {name: f"[{n} x {k}] split over {world} ranks by input feature" for name, (n, k) in shapes.items()},
            "tokens": list(ntoks), "mode": ar.mode, "consumer_side": arc.publish_only,
            "max_rel_err": {key: worst[key] for key in checked},
            "max_abs_diff_between_ranks": worst["ranks_differ"],
            "tolerance": tol,
            "ok": all(worst[key] <= tol for key in checked) and worst["ranks_differ"] == 0.0 and t[-1].item() == 0,
            "us_per_call_32_tokens": us,
            "timing_basis": "each rank's whole shard in HBM; CUDA graph of 10 calls, events, max over ranks",
            "reference": "torch F.linear(x.float(), W.float()) of the full weight on rank 0's host cores; "
                         "RMSNorm of the 16-bit residual sum in FP32"}


def run_linear(args, torch, rank, world):
    from directaccesskernel_b200 import runtime

    prefill, tokens, ratios = linear_sweep(args)
    tp = world > 1
    hbm_gbs, peak_kind = measured_peaks()
    tflops, tflops_kind = measured_tensor_tflops()
    dma_gbs, tma_host_gbs = host_link_probe(torch, runtime, world)
    host_gbs = max(dma_gbs, tma_host_gbs)
    hbm_read_gbs = hbm_read_probe(torch, runtime)

    host_frac, host_by_rank = None, [host_gbs]
    if tp:
        # Each rank streams its own shard over its own host link; all links are
        # measured at once.  Host rows go to the ranks in proportion to their
        # concurrent GPU-initiated read bandwidth, so that all host streams end
        # together; the mean host fraction per layer stays the sweep's ratio.
        bw = torch.tensor([tma_host_gbs, host_gbs], dtype=torch.float64, device="cuda")
        parts = [torch.zeros_like(bw) for _ in range(world)]
        torch.distributed.all_gather(parts, bw)
        tma_by_rank = [float(t[0]) for t in parts]
        host_by_rank = [float(t[1]) for t in parts]
        host_frac = {r: (r if (args.no_balance or r in (0.0, 1.0)) else balanced_host_fractions(r, tma_by_rank)[rank])
                     for r in ratios}

    built = build_layers(torch, tokens, ratios, seed=0 if tp else rank, rank=rank, world=world,
                         host_frac=host_frac, keep_weights=(rank == 0))
    layers, weights = built if rank == 0 else (built, None)
    gen = torch.Generator(device="cuda").manual_seed(1234 if tp else 1234 + rank)
    x_dev = {(m, k): torch.randn(m, 1, k, generator=gen, device="cuda").half()
             for m in tokens for k in sorted({l["k"] for l in layers})}
    calls = [(l, m) for m in tokens for l in layers]

    # The device-timed region replays CUDA graphs, as the reference's decode
    # loop does (benchmark_opt.py:344-357): one graph per step for `value`,
    # and one graph per layer call, replayed back to back with events between
    # them, for the per-launch roofline breakdown.  Under tensor parallelism
    # each call's all-gather (NCCL) is captured in the same graphs.
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(1, args.warmup)):
            for (l, m) in calls:
                l["mod"](x_dev[(m, l["k"])])
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph):
        for (l, m) in calls:
            l["mod"](x_dev[(m, l["k"])])
    call_graphs = []
    for (l, m) in calls:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            l["mod"](x_dev[(m, l["k"])])
        call_graphs.append(g)
    # One graph per offload ratio (its 16 layer calls back to back), for the
    # per-ratio breakdown with the same launch overlap as the step graph.
    ratio_graphs = {}
    for r in ratios:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for (l, m) in calls:
                if l["ratio"] == r:
                    l["mod"](x_dev[(m, l["k"])])
        ratio_graphs[r] = g
    stream = torch.cuda.current_stream()

    # ---- device-resident timing (value): whole-step graphs back to back
    for _ in range(args.warmup):
        step_graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        t0.record(stream)
        for _ in range(args.steps):
            step_graph.replay()
        t1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    total_ms = t0.elapsed_time(t1)
    clock = clocks.summary()

    # ---- per-launch durations: per-call graphs, events between them
    launch_ms = [0.0] * len(calls)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(calls) + 1)] for _ in range(args.steps)]
    for s in range(args.steps):
        evs[s][0].record(stream)
        for i, g in enumerate(call_graphs):
            g.replay()
            evs[s][i + 1].record(stream)
    torch.cuda.synchronize()
    for s in range(args.steps):
        for i in range(len(calls)):
            launch_ms[i] += evs[s][i].elapsed_time(evs[s][i + 1])
    ratio_ms = {r: 0.0 for r in ratios}
    rev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(ratios) + 1)] for _ in range(args.steps)]
    for s in range(args.steps):
        rev[s][0].record(stream)
        for j, r in enumerate(ratios):
            ratio_graphs[r].replay()
            rev[s][j + 1].record(stream)
    torch.cuda.synchronize()
    for s in range(args.steps):
        for j, r in enumerate(ratios):
            ratio_ms[r] += rev[s][j].elapsed_time(rev[s][j + 1])
    status = runtime.device_status()
    if status != 0:
        raise RuntimeError(f"device error word {status} after the timed region")
    # Graphs that hold NCCL calls are released before the process group goes.
    g = None
    del g, step_graph, call_graphs, ratio_graphs
    torch.cuda.synchronize()

    # ---- end to end through the module API with host buffers (e2e).  Every
    # step uploads its distinct activations from pinned host memory in one
    # copy, runs the layers eagerly through the module API, and reads every
    # layer's output back to pinned host memory on a side stream as soon as
    # the layer is done, so the read-backs overlap the later layers instead of
    # sitting between them.
    keys = sorted(x_dev)
    offs, total = {}, 0
    for key in keys:
        offs[key] = total
        total += x_dev[key].numel()
    x_host_all = torch.empty(total, dtype=torch.float16).pin_memory()
    for key in keys:
        x_host_all[offs[key]:offs[key] + x_dev[key].numel()].copy_(x_dev[key].reshape(-1).cpu())
    x_step = torch.empty(total, dtype=torch.float16, device="cuda")
    x_in = {key: x_step[offs[key]:offs[key] + x_dev[key].numel()].view(x_dev[key].shape) for key in keys}
    y_host = [torch.empty(m, 1, l["n"], dtype=torch.float16).pin_memory() for (l, m) in calls]
    h2d = world * total * 2
    d2h = world * sum(y.numel() * 2 for y in y_host)
    copy_stream = torch.cuda.Stream()
    done = [torch.cuda.Event() for _ in calls]

    def step_e2e():
        x_step.copy_(x_host_all, non_blocking=True)
        for i, (l, m) in enumerate(calls):
            y = l["mod"](x_in[(m, l["k"])])
            done[i].record(stream)
            copy_stream.wait_event(done[i])
            with torch.cuda.stream(copy_stream):
                y_host[i].copy_(y, non_blocking=True)
            y.record_stream(copy_stream)
        stream.wait_stream(copy_stream)

    for _ in range(args.warmup):
        step_e2e()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_e2e()
    e1.record(stream)
    torch.cuda.synchronize()
    # The read-backs are the layers' outputs.
    for i, (l, m) in enumerate(calls[:4]):
        if not torch.isfinite(y_host[i].float()).all():
            raise RuntimeError("e2e: a read-back output is not finite")
    e2e_ms = e0.elapsed_time(e1)

    # ---- parity of the outputs of one eager pass (all ranks take part in the
    # all-gathers; rank 0 checks the gathered outputs on the host)
    outputs = [l["mod"](x_dev[(m, l["k"])]).clone() for (l, m) in calls]
    torch.cuda.synchronize()
    parity = linear_parity(torch, layers, calls, outputs, weights, x_dev) if rank == 0 else None
    del outputs
    # Under tensor parallelism, the row-parallel layers' all-reduce as well.
    row_parallel = row_parallel_check(torch, rank, world) if tp and not args.no_row_parallel else None

    # ---- reduce over ranks (max time, summed bytes)
    w_bytes_step = sum(l["w_bytes"] for (l, m) in calls)
    kernel_ms = sum(launch_ms)
    times = torch.tensor([total_ms, kernel_ms, e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(times, op=torch.distributed.ReduceOp.MAX)
    total_ms, kernel_ms, e2e_ms = times.tolist()

    # Roofline per layer call: max((1-r)W/HBM, rW/host, 2MNK/tensor peak), with
    # x and y bytes riding with HBM; the compute term only binds for
    # prefill-sized M.  Under tensor parallelism each rank's term uses its own
    # shard, host rows and concurrently measured host link, plus the bytes the
    # all-gather brings in over NVLink; a call is bound by its slowest rank.
    per_call = []
    for (l, m) in calls:
        which, t_s = layer_roofline(m, l["rank_n"], l["k"], l["host_bytes"], hbm_gbs, host_gbs, tflops)
        if tp:
            t_nv = (world - 1) / world * m * l["n"] * 2 / (NVLINK_GBS * 1e9)
            if t_nv > t_s:
                which, t_s = "nvlink", t_nv
        per_call.append((which, t_s * 1e3))
    roof_t = torch.tensor([t for (_, t) in per_call], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(roof_t, op=torch.distributed.ReduceOp.MAX)
    roof_call = roof_t.tolist()
    roof_ms = 0.0
    alg_bytes = 0
    dram_bytes = 0.0
    per_ratio = {}
    bound_ms = {"hbm": 0.0, "host": 0.0, "tensor": 0.0, "nvlink": 0.0}
    for i, (l, m) in enumerate(calls):
        io = (m * l["k"] + m * l["n"]) * 2
        dram_bytes += (l["rank_n"] * l["k"] * 2 - l["host_bytes"] + io) * DRAM_PER_DEVICE_BYTE
        t_roof = roof_call[i]
        bound_ms[per_call[i][0]] += t_roof * args.steps
        roof_ms += t_roof * args.steps
        alg_bytes += l["w_bytes"] + io
        pr = per_ratio.setdefault(l["ratio"], {"bytes": 0, "ms": ratio_ms[l["ratio"]], "roof_ms": 0.0,
                                               "isolated_ms": 0.0})
        pr["bytes"] += l["w_bytes"] * args.steps
        pr["isolated_ms"] += launch_ms[i]
        pr["roof_ms"] += t_roof * args.steps
    # Achieved bandwidth averaged over the timed launches of the step graph
    # (total algorithmic bytes of the job / device time).
    achieved = alg_bytes * args.steps / (total_ms * 1e-3) / 1e9
    peak_eff = alg_bytes * args.steps / (roof_ms * 1e-3) / 1e9
    value = w_bytes_step * args.steps / (total_ms * 1e-3) / 1e9
    e2e = w_bytes_step * args.steps / (e2e_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_linear(tokens, ratios)

    details = [{"layer": l["name"], "m": m, "ratio": l["ratio"], "rank_ratio": l["rank_ratio"],
                "ms": launch_ms[i] / args.steps, "gbs": l["w_bytes"] / (launch_ms[i] / args.steps * 1e-3) / 1e9}
               for i, (l, m) in enumerate(calls)]
    if args.details and rank == 0:
        Path(args.details).write_text(json.dumps(details, indent=1))
    metric, config = linear_metric_config(prefill, tokens, ratios, world)
    tp_info = None
    if tp:
        tp_info = {"host_fraction_per_rank": {str(r): round(f, 4) for r, f in host_frac.items()},
                   "host_fraction_basis": "rank 0's share; shares are proportional to each rank's concurrent "
                                          "GPU-initiated host read bandwidth, mean over ranks = r",
                   "host_link_gbs_per_rank": [round(v, 2) for v in host_by_rank]}
    line = {
        "metric": metric,
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if tp else "weak",
        "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)", "data": "synthetic N(0,0.02) weights, N(0,1) activations",
        "config": config,
        "roofline": {"bound": "tensor" if bound_ms["tensor"] > bound_ms["hbm"] + bound_ms["host"] else "hbm",
                     "achieved": round(achieved, 2), "peak": round(peak_eff, 2), "unit": "GB/s",
                     "frac": round(achieved / peak_eff, 4),
                     "traffic": round(dram_bytes / len(calls)),
                     "traffic_basis": "DRAM bytes per launch on rank 0, step average: ncu dram read+write = "
                                      f"{DRAM_PER_DEVICE_BYTE} x device-tier bytes on full-size captures; the "
                                      "host tier's bytes cross PCIe, so traffic < algorithmic bytes "
                                      f"({round(alg_bytes / len(calls))} per launch)",
                     "peak_model": "combined HBM + host-link (+ tensor, + NVLink all-gather under tp) roofline, sum "
                                   "over layers of the slowest rank's max((1-r)W/HBM, rW/host, 2MNK/tensor peak, "
                                   "gathered bytes/NVLink)",
                     "bound_ms_by_term": {k: round(v, 4) for k, v in bound_ms.items()},
                     "tensor_tflops": tflops, "tensor_peak_kind": tflops_kind,
                     "hbm_gbs": hbm_gbs, "hbm_peak_kind": peak_kind, "host_link_gbs": round(host_gbs, 2),
                     "host_link_dma_gbs": round(dma_gbs, 2), "host_link_tma_probe_gbs": round(tma_host_gbs, 2),
                     "hbm_read_probe_gbs": round(hbm_read_gbs, 1),
                     "per_ratio": {str(r): {"gbs": round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 2),
                                            "frac": round(v["roof_ms"] / v["ms"], 4),
                                            "isolated_launch_frac": round(v["roof_ms"] / v["isolated_ms"], 4)}
                                   for r, v in per_ratio.items()},
                     "timing": "achieved = algorithmic bytes / device time of the step graph; per_ratio from one "
                               "graph per ratio; isolated_launch_frac from single-launch graphs with events between"},
        "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "method": "per step: one copy of the step's distinct activations from pinned host memory, every "
                          "layer through the module API (eager), every layer's output read back to pinned host "
                          "memory on a side stream as soon as the layer is done"},
        "gpu_launches": world * sum(-(-m // (2 * MMA_MAX_TOKENS if m > MMA_MAX_TOKENS else MMA_MAX_TOKENS))
                                    for (l, m) in calls) * args.steps,
        "clocks": clock,
        "parity": parity,
    }
    if tp:
        line["tp"] = tp_info
        if row_parallel is not None:
            line["row_parallel"] = row_parallel
        line["roofline"]["nvlink_gbs"] = NVLINK_GBS
        line["roofline"]["host_link_basis"] = "each rank's own link, all ranks streaming at once"
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def run_plan_sweep(args, torch, rank, world):
    """Launch-plan sweep of the HBM-only (r = 0) Llama-3-8B layers, one GPU: the
    automatic plan and explicit (dev_ctas, dev_ksplit) plans, each timed two
    ways.  Chained: a CUDA graph of 8 calls on distinct weight copies (more than
    L2), so the overlap of consecutive launches counts; per call = graph / 8.
    Isolated: a graph of one call.  One JSON record per plan goes to
    ``--details``; the line summarises the automatic plan against the best."""
    from directaccesskernel_b200 import runtime

    tp8 = args.sweep_shapes == "llama70b-tp8"
    shapes = LLAMA70B_TP8 if tp8 else LLAMA8B
    tokens = [int(t) for t in args.tokens.split(",")] if args.tokens else ([32] if tp8 else list(TOKENS))
    copies, reps = 8, max(3, args.steps)
    stream = torch.cuda.current_stream()

    def timed(graph):
        for _ in range(max(1, args.warmup)):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    records = []
    for name, (n, k) in shapes.items():
        ws = [(torch.randn(k, n, device="cuda") * 0.02).half() for _ in range(copies)]
        for m in tokens:
            x = torch.randn(m, k, device="cuda").half()
            ys = [torch.empty(m, n, device="cuda", dtype=torch.float16) for _ in range(copies)]
            kss = (1, 2, 4) if m > 2 else (1, 2, 4, 8)
            plans = [(0, 0)] + [(c, ks) for ks in kss for c in (32, 48, 64, 96, 128, 144, 148)
                                if 1 <= c // ks <= (n + 63) // 64]
            for (c, ks) in plans:
                def call(i):
                    runtime.linear_split(x, ys[i], None, ws[i], dev_ctas=c, dev_ksplit=ks)

                for i in range(copies):
                    call(i)
                side = torch.cuda.Stream()
                side.wait_stream(stream)
                with torch.cuda.stream(side):
                    chain, one = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
                    with torch.cuda.graph(chain):
                        for i in range(copies):
                            call(i)
                    with torch.cuda.graph(one):
                        call(0)
                stream.wait_stream(side)
                chained, isolated = timed(chain) / copies, timed(one)
                del chain, one
                records.append({"shape": name, "m": m, "ctas": c, "ksplit": ks, "chained_us": round(chained * 1e3, 3),
                                "isolated_us": round(isolated * 1e3, 3),
                                "chained_tbs": round(2 * n * k / (chained * 1e-3) / 1e12, 3)})
        del ws
        torch.cuda.empty_cache()
    if runtime.device_status() != 0:
        raise RuntimeError("device error word set during the plan sweep")
    if args.details:
        Path(args.details).write_text("\n".join(json.dumps(r) for r in records) + "\n")
    auto = {(r["shape"], r["m"]): r["chained_us"] for r in records if r["ctas"] == 0}
    best = {}
    for r in records:
        key = (r["shape"], r["m"])
        best[key] = min(best.get(key, float("inf")), r["chained_us"])
    hbm_gbs, peak_kind = measured_peaks()
    roof_us = sum(2 * n * k / (hbm_gbs * 1e9) * 1e6 for (n, k) in shapes.values()) * len(tokens)
    return {"metric": "HBM-only linear launch plans: chained microseconds per call, automatic vs best explicit plan",
            "value": round(sum(auto.values()), 2), "unit": "us (sum over shapes x M, automatic plan)", "n_gpus": 1,
            "steps": reps, "warmup": args.warmup, "higher_is_better": False,
            "best_explicit_us": round(sum(best.values()), 2), "hbm_roofline_us": round(roof_us, 2),
            "hbm_gbs": hbm_gbs, "hbm_peak_kind": peak_kind, "plans": len(records),
            "config": {"workload": (f"{'one TP8 rank of Llama-3-70B' if tp8 else 'Llama-3-8B'} qkv/o/gate_up/down in "
                                    f"HBM x M{tokens}; {copies} weight copies per chain (more than L2)")}}


def run_read_ceiling(args, torch, rank, world):
    """What a launch-separated HBM stream reaches on the four Llama-3-8B weight
    sizes, one GPU: the library's bandwidth probe (TMA bulk reads into a
    shared-memory ring, a checksum as the only output) at several launch
    shapes, against the HBM-only (r = 0) linear kernels at M = 1 on the same
    bytes, timed the same two ways.  Isolated: one launch at a time, L2 flushed
    before each.  Chained: the four layers as one CUDA graph of four launches,
    L2 flushed before the graph; each line of the graph reads its own bytes."""
    from directaccesskernel_b200 import runtime

    hbm_gbs, peak_kind = measured_peaks()
    stream = torch.cuda.current_stream()
    flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    # The linear entry point takes the transposed weight, [K, N] (the layout the modules keep).
    weights = {name: (torch.randn(k, n, device="cuda") * 0.02).half() for name, (n, k) in LLAMA8B.items()}
    xs = {name: torch.randn(1, k, device="cuda").half() for name, (n, k) in LLAMA8B.items()}
    ys = {name: torch.empty(1, n, device="cuda", dtype=torch.float16) for name, (n, k) in LLAMA8B.items()}
    total = sum(w.numel() * 2 for w in weights.values())
    sink = torch.zeros(1, dtype=torch.int32, device="cuda")
    reps = max(3, args.steps)

    def graph_of(calls):
        for c in calls:
            c()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side), torch.cuda.graph(g):
            for c in calls:
                c()
        stream.wait_stream(side)
        return g

    def timed(graph):
        best = float("inf")
        for _ in range(max(1, args.warmup)):
            graph.replay()
        for _ in range(reps):
            flush.add_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1e-3)
        return best

    def measure(make_call):
        calls = [make_call(name) for name in LLAMA8B]
        iso = sum(timed(graph_of([c])) for c in calls)
        chained = timed(graph_of(calls))
        return {"isolated_frac": round(total / iso / 1e9 / hbm_gbs, 3),
                "chained_frac": round(total / chained / 1e9 / hbm_gbs, 3),
                "chained_us": round(chained * 1e6, 2)}

    results = []
    for ctas, stages, chunk in ((runtime.NUM_SMS, 6, 32768), (runtime.NUM_SMS, 12, 16384),
                                (2 * runtime.NUM_SMS, 6, 16384), (runtime.NUM_SMS, 3, 65536)):
        r = measure(lambda name, c=ctas, s=stages, ch=chunk: (lambda: runtime.probe_stream_read(
            weights[name].view(torch.uint8).view(-1), c, s, ch, sink=sink)))
        results.append({"kernel": "probe_read", "ctas": ctas, "stages": stages, "chunk_bytes": chunk, **r})
    lin = measure(lambda name: (lambda: runtime.linear_split(xs[name], ys[name], None, weights[name])))
    results.append({"kernel": "linear (automatic plan), M = 1, r = 0", **lin})
    if runtime.device_status() != 0:
        raise RuntimeError("device error word set during the read-ceiling run")
    best_probe = max(r["chained_frac"] for r in results if r["kernel"] == "probe_read")
    return {"metric": "HBM read ceiling of launch-separated streams: fraction of measured HBM peak, four "
                      "Llama-3-8B weight sizes as four launches in one CUDA graph",
            "value": best_probe, "unit": "fraction of hbm_gbs", "n_gpus": 1, "steps": reps, "warmup": args.warmup,
            "higher_is_better": True, "linear_chained_frac": lin["chained_frac"],
            "linear_isolated_frac": lin["isolated_frac"], "shapes": results, "hbm_gbs": hbm_gbs,
            "hbm_peak_kind": peak_kind, "weight_bytes": total,
            "config": {"workload": "Llama-3-8B qkv/o/gate_up/down weight bytes (436 MB), L2 flushed before each "
                                   "timed graph; best of the timed replays"}}


class CpuLinearSweep:
    """The sweep's layer calls computed on the host cores, for the CPU baseline
    and the reference arm.  ``impl`` "torch" is the reference's own computation
    of a layer, torch F.linear on FP32 copies (benchmark_linear.py:121-123 runs
    nn.Linear); "port" is the oracle's numpy restatement.  Weights and inputs
    are built once, before anything is timed.  One pass computes every layer
    call of one step (shapes x M x ratios; the host computation does not depend
    on the offload ratio), and only whole passes are timed."""

    def __init__(self, tokens, ratios, impl: str = "torch", seed: int = 0):
        import numpy as np

        self.impl, self.tokens, self.ratios = impl, list(tokens), list(ratios)
        self.threads = os.cpu_count()
        rng = np.random.default_rng(seed)
        self.w, self.x = {}, {}
        for name, (n, k) in LLAMA8B.items():
            w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
            for m in self.tokens:
                self.x[(name, m)] = rng.standard_normal((m, k), dtype=np.float32)
            self.w[name] = w
        if impl == "torch":
            import torch

            torch.set_num_threads(self.threads)
            self.w = {k: torch.from_numpy(v) for k, v in self.w.items()}
            self.x = {k: torch.from_numpy(v) for k, v in self.x.items()}
        self.bytes_per_pass = len(self.ratios) * len(self.tokens) * sum(2 * n * k for (n, k) in LLAMA8B.values())
        self.calls_per_pass = len(self.ratios) * len(self.tokens) * len(LLAMA8B)

    def one_pass(self):
        if self.impl == "torch":
            import torch.nn.functional as F

            for _ in self.ratios:
                for m in self.tokens:
                    for name in LLAMA8B:
                        F.linear(self.x[(name, m)], self.w[name])
        else:
            import numpy as np

            import oracle  # the checker, timed here as the CPU baseline

            for _ in self.ratios:
                for m in self.tokens:
                    for name in LLAMA8B:
                        oracle.linear(self.x[(name, m)], self.w[name], acc=np.float32)

    def timed_passes(self, passes: int, warmup: int = 1) -> list[float]:
        for _ in range(warmup):
            self.one_pass()
        times = []
        for _ in range(passes):
            t = time.perf_counter()
            self.one_pass()
            times.append(time.perf_counter() - t)
        return times

    def sample(self) -> str:
        what = ("torch F.linear(x, W) on FP32 copies (the reference's computation, benchmark_linear.py:121-123)"
                if self.impl == "torch" else "the oracle's numpy FP32 x @ W^T")
        return (f"{what}: whole passes over the {self.calls_per_pass} layer calls of one step "
                f"(4 Llama-3-8B shapes x M{self.tokens} x {len(self.ratios)} ratios; host time does not depend on "
                f"the ratio), weights built before timing, {self.threads} threads; GB/s of fp16 weight bytes")


def cpu_baseline_linear(tokens, ratios, passes: int = 3, warmup: int = 3):
    """cpu_baseline of the GPU arm: the median of whole timed passes of the
    reference's computation (torch F.linear, FP32) on all host cores, after
    ``warmup`` untimed passes (as the reference arm takes), with the oracle
    port's figure beside it."""
    out = {}
    for impl in ("torch", "port"):
        sweep = CpuLinearSweep(tokens, ratios, impl)
        times = sweep.timed_passes(passes, warmup=warmup)
        out[impl] = (sweep.bytes_per_pass / statistics.median(times) / 1e9, sweep, len(times))
        del sweep
    v, sweep, n = out["torch"]
    return {"value": round(v, 3), "unit": "GB/s", "cores": sweep.threads, "kind": "reference",
            "sample": sweep.sample() + f"; median of {n} passes",
            "port_value": round(out["port"][0], 3), "port_kind": "port (numpy oracle, same passes)"}


def run_attention(args, torch, rank, world):
    """B=8, 32/8 heads, D=128, ctx 32768, 16-token pages, 50% on host."""
    from directaccesskernel_b200 import runtime
    from directaccesskernel_b200.attention import auto_split_size, decode_paged

    hbm_gbs, peak_kind = measured_peaks()
    dma_gbs, tma_host_gbs = host_link_probe(torch, runtime, world)
    host_gbs = max(dma_gbs, tma_host_gbs)
    B, Hq, Hkv, S, P = 8, 32, 8, 32768, 16
    g = torch.Generator(device="cuda").manual_seed(rank)
    npg = B * S // P
    perm = torch.randperm(npg, generator=torch.Generator().manual_seed(0))
    host_pages, dev_pages = perm[: npg // 2], perm[npg // 2:]
    kd = torch.randn(len(dev_pages), Hkv, P, 128, generator=g, device="cuda", dtype=torch.float16)
    vd = torch.randn(len(dev_pages), Hkv, P, 128, generator=g, device="cuda", dtype=torch.float16)
    kh = torch.randn(len(host_pages), Hkv, P, 128, generator=g, device="cuda", dtype=torch.float16).cpu().pin_memory()
    vh = torch.randn(len(host_pages), Hkv, P, 128, generator=g, device="cuda", dtype=torch.float16).cpu().pin_memory()
    table = torch.empty(npg, dtype=torch.int32)
    table[host_pages] = -1 - torch.arange(len(host_pages), dtype=torch.int32)
    table[dev_pages] = torch.arange(len(dev_pages), dtype=torch.int32)
    table = table.view(B, S // P).cuda()
    seq = torch.full((B,), S, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq, 128, generator=g, device="cuda", dtype=torch.float16)
    split = auto_split_size(B, Hkv, S)
    ns = (S + split - 1) // split
    out = torch.empty(B, Hq, 128, dtype=torch.float16, device="cuda")
    po = torch.empty(B, Hq, ns, 128, dtype=torch.float32, device="cuda")
    pml = torch.empty(B, Hq, ns, 2, dtype=torch.float32, device="cuda")
    scale = 1.0 / math.sqrt(128)

    def step():
        decode_paged(q, kd, vd, kh, vh, table, seq, scale, split, out=out, partial_o=po, partial_ml=pml)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    kv_bytes = 2 * B * Hkv * S * 128 * 2
    host_bytes = kv_bytes // 2

    # End to end: the query comes from pinned host memory and the output goes back
    # to it every step.
    q_host = q.cpu().pin_memory()
    o_host = torch.empty_like(out, device="cpu").pin_memory()

    def step_e2e():
        q.copy_(q_host, non_blocking=True)
        step()
        o_host.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        step_e2e()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        step_e2e()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_attention()
    roof_ms = max((kv_bytes - host_bytes) / (hbm_gbs * 1e9), host_bytes / (host_gbs * 1e9)) * 1e3
    achieved = kv_bytes * args.steps / (ms * 1e-3) / 1e9
    return {
        "metric": "split-KV decode attention KV GB/s", "value": round(world * achieved, 2), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 softmax)",
        "data": "synthetic N(0,1) K/V/Q",
        "config": {"workload": "BASELINE config 3: B8 Hq32 Hkv8 D128 ctx32768 16-token pages 50% host",
                   "split_size": split, "l2": "1 GiB of KV per step exceeds L2"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2),
                     "peak": round(kv_bytes / (roof_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "frac": round(roof_ms * args.steps / ms, 4),
                     "traffic": round((kv_bytes - host_bytes) * ATTN_DRAM_PER_DEVICE_BYTE),
                     "traffic_basis": "ncu dram read+write of one full-size config-3 launch: 541.6 MB for 536.9 MB "
                                      "of device-resident K/V",
                     "peak_model": "max(device KV / HBM, host KV / host link)", "hbm_gbs": hbm_gbs,
                     "hbm_peak_kind": peak_kind, "host_link_gbs": round(host_gbs, 2)},
        "e2e": {"value": round(world * kv_bytes * args.steps / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": q_host.numel() * 2, "d2h_bytes_per_step": o_host.numel() * 2},
        "gpu_launches": 2 * args.steps, "clocks": clocks.summary(),
        **({"cpu_baseline": cpu} if cpu is not None else {}),
    }


def cpu_baseline_attention(budget_s: float = 15.0):
    """The oracle port of the attention (numpy FP32 softmax attention per GQA
    group, BLAS matrix products on all host threads) on a bounded sample of
    config 3: whole sequences of 32768 tokens, all 8 KV heads, one at a time."""
    import numpy as np

    import oracle.attention as oatt

    rng = np.random.default_rng(0)
    Hq, Hkv, S, D = 32, 8, 32768, 128
    k = rng.standard_normal((1, Hkv, S, D), dtype=np.float32)
    v = rng.standard_normal((1, Hkv, S, D), dtype=np.float32)
    t_total, seqs = 0.0, 0
    while t_total < budget_s and seqs < 64:
        q = rng.standard_normal((1, Hq, 1, D), dtype=np.float32)
        t = time.perf_counter()
        oatt.decode_attention_grouped(q, k, v, 1.0 / math.sqrt(D))
        t_total += time.perf_counter() - t
        seqs += 1
    kv_fp16 = 2 * Hkv * S * D * 2 * seqs
    return {"value": round(kv_fp16 / t_total / 1e9, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{seqs} whole sequences (ctx {S}, Hq {Hq} / Hkv {Hkv}, D {D}) of config 3; "
                      "fp16 KV bytes / numpy FP32 time"}


# ------------------------------------------------------------ opt66b decode
OPT66B_LINEARS_PER_LAYER = 6  # q, k, v, out_proj, fc1, fc2


def run_opt66b(args, torch, rank, world):
    """OPT-66B architecture (random N(0, 0.02) fp16 weights, 131.4 GB)
    under an HBM weight budget; the placement puts the rest of the decoder linears in
    pinned host memory.  Batch 1, a random 512-token prompt, greedy decode with one
    CUDA graph per step (benchmark_opt.py:137-460).  Metric: decode tokens/s."""
    if world > 1:
        raise SystemExit("the opt66b workload runs on one GPU (BASELINE config 4); it pins ~35 GB of host "
                         "memory per process")
    from directaccesskernel_b200 import decode, runtime

    hbm_gbs, peak_kind = measured_peaks()
    dma_gbs, tma_host_gbs = host_link_probe(torch, runtime, world)
    host_gbs = max(dma_gbs, tma_host_gbs)
    cfg = decode.opt_config("opt-66b")
    budget_gb = 96.0 if args.hbm_budget_gb is None else args.hbm_budget_gb
    budget = int(budget_gb * 1e9)
    t0 = time.perf_counter()
    model, stats = decode.build_offloaded_model(cfg, linear_type="horizontal", hbm_budget_bytes=budget, seed=rank)
    build_s = time.perf_counter() - t0
    B, L = 1, args.prompt_len
    W, K = max(3, args.warmup), args.steps
    prompt = decode.random_prompt(B, L, cfg.vocab_size, seed=0)
    dec = decode.GreedyDecoder(model, B, L + W + 2 * K + 8, graph=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        res = dec.generate(prompt, W + K, warmup_steps=W)
    tbt = res.tbt_ms
    model_bytes = stats.host_bytes + stats.device_bytes
    roof_ms = decode.decode_roofline_ms(stats, hbm_gbs, host_gbs)
    status = runtime.device_status()
    if status != 0:
        raise RuntimeError(f"device error word {status} after the timed region")

    # End to end: every step the token goes to pinned host memory and comes back as
    # the next step's input, as a serving loop that streams tokens out does.
    tok_host = torch.empty(B, 1, dtype=torch.long).pin_memory()
    tok_host.copy_(res.tokens[:, -1:])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.inference_mode():
        e0.record()
        for _ in range(K):
            dec.ids.copy_(tok_host, non_blocking=True)
            logits = dec.step()
            nxt = torch.argmax(logits, dim=-1)
            tok_host.copy_(nxt[:, None], non_blocking=True)
            torch.cuda.current_stream().synchronize()
            dec.advance(logits, forced=nxt)
        e1.record()
        torch.cuda.synchronize()
    e2e_tbt = e0.elapsed_time(e1) / K

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline_opt66b()
    n_layers = cfg.num_hidden_layers
    return {
        "metric": "decode tokens/s (OPT-66B arch, HBM weight budget)", "value": round(B * 1e3 / tbt, 4),
        "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(tbt, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
        "data": "synthetic: random N(0,0.02) weights, random prompt ids",
        "config": {"workload": f"BASELINE config 4: OPT-66B arch, HBM budget {budget_gb:g} GB, batch {B}, "
                               f"prompt {L}, greedy decode", "model_bytes": model_bytes,
                   "host_bytes": stats.host_bytes, "device_bytes": stats.device_bytes,
                   "weight_offload_ratio": round(stats.actual_offload_ratio, 4), "build_s": round(build_s, 1),
                   "prefill_ms": round(res.prefill_ms, 1), "l2": "131 GB of weights per step exceed L2",
                   "timing": "CUDA events around each graph replay of one decode step"},
        "roofline": {"bound": "hbm", "achieved": round(model_bytes / (tbt * 1e-3) / 1e9, 2),
                     "peak": round(model_bytes / (roof_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "frac": round(roof_ms / tbt, 4),
                     "traffic": round(stats.device_bytes * DRAM_PER_DEVICE_BYTE),
                     "traffic_basis": "per decode step: device-resident weight bytes x the DRAM/device-byte ratio "
                                      "of the linear captures",
                     "peak_model": "max(device weight bytes / HBM, host weight bytes / host link) per step",
                     "hbm_gbs": hbm_gbs, "hbm_peak_kind": peak_kind, "host_link_gbs": round(host_gbs, 2),
                     "host_link_dma_gbs": round(dma_gbs, 2), "host_link_tma_probe_gbs": round(tma_host_gbs, 2)},
        "e2e": {"value": round(B * 1e3 / e2e_tbt, 4), "unit": "tokens/s", "h2d_bytes_per_step": 8 * B,
                "d2h_bytes_per_step": 8 * B},
        "gpu_launches": OPT66B_LINEARS_PER_LAYER * n_layers * K, "clocks": clocks.summary(),
        **({"cpu_baseline": cpu} if cpu is not None else {}),
    }


def run_llama70b(args, torch, rank, world):
    """Llama-3-70B architecture, tensor-parallel over the
    torchrun ranks, batch 32, context 16384 (random KV standing in for the
    prefill), a per-GPU HBM budget (60 GB) that puts the same fraction of each
    rank's weights and KV pages in its pinned host memory.  One step = one
    greedy decode step of all sequences (one CUDA graph, NCCL all-reduce after
    o and down).  ``--layers`` and ``--host-fraction`` give the reduced-depth,
    fixed-fraction variant whose host bytes fit the box at every TP size."""
    import psutil

    from directaccesskernel_b200 import decode, runtime
    from directaccesskernel_b200.llama_tp import LlamaShape, TPLlamaDecoder, budget_fraction

    hbm_gbs, peak_kind = measured_peaks()
    dma_gbs, tma_host_gbs = host_link_probe(torch, runtime, world)
    host_gbs = max(dma_gbs, tma_host_gbs)
    cfg = decode.llama_config("llama-3-70b", num_hidden_layers=args.layers)
    shape = LlamaShape.from_config(cfg)
    emulated = args.rank_of_tp if world == 1 and args.rank_of_tp > 1 else 1
    if emulated > 1:
        shape = rank_shape(shape, emulated)
    B, ctx = args.batch, args.ctx
    W, K = max(3, args.warmup), args.steps
    # Room for every token the run appends: warm-up, timed and end-to-end steps,
    # the profiled step, and the capture's warm-up step (undone, but written).
    max_ctx = ctx + W + 2 * K + 4
    budget_gb = 60.0 if args.hbm_budget_gb is None else args.hbm_budget_gb
    frac = (args.host_fraction if args.host_fraction is not None
            else budget_fraction(shape, world, B, max_ctx, int(budget_gb * 1e9)))
    per_rank_total = shape.weight_bytes_per_rank(world) + shape.kv_bytes_per_rank(world, B, max_ctx)
    host_need = frac * per_rank_total * world
    # The ranks share the box's host-memory bandwidth unevenly; give each rank a
    # share of the host bytes proportional to its concurrently measured
    # GPU-initiated read bandwidth, so that all host streams finish together.
    fracs = [frac] * world
    if world > 1 and frac > 0 and not args.no_balance:
        bw = torch.tensor([tma_host_gbs], dtype=torch.float64, device="cuda")
        allbw = torch.empty(world, dtype=torch.float64, device="cuda")
        torch.distributed.all_gather_into_tensor(allbw, bw)
        lo = max(0.0, 1.0 - budget_gb * 1e9 / per_rank_total)
        fracs = balanced_host_fractions(frac, allbw.tolist(), lo)
    my_frac = fracs[rank]
    ram = psutil.virtual_memory().total
    if host_need > 0.75 * ram:
        raise SystemExit(f"llama70b at TP{world}: {host_need / 1e9:.0f} GB of pinned host memory needed, more than "
                         f"3/4 of the box's {ram / 1e9:.0f} GB; use --layers / --host-fraction")
    t0 = time.perf_counter()
    fused = world > 1 and not args.nccl_allreduce
    dec = TPLlamaDecoder(shape, batch=B, max_ctx=max_ctx, weight_offload=my_frac, kv_host_fraction=my_frac,
                         fused_allreduce=fused)
    dec.init_random(seed=0)
    dec.fill_kv_random(ctx, seed=1)
    g = torch.Generator().manual_seed(3)
    dec.ids.copy_(torch.randint(0, shape.vocab, (B,), generator=g).cuda())
    build_s = time.perf_counter() - t0
    # With the fused reduction available, the decoder times one step each way
    # (consumer-side reduction, linear + NCCL) and keeps the faster.
    dec.capture(choose_allreduce=fused)
    fused = dec.use_fused
    for _ in range(W):
        dec.step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        e0.record()
        for _ in range(K):
            dec.step()
        e1.record()
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = e0.elapsed_time(e1)
    # End to end: every step the new tokens go to pinned host memory and the host
    # waits for them, as a serving loop that streams tokens out does.
    tok_host = torch.empty(B, dtype=torch.long).pin_memory()
    torch.cuda.synchronize()
    e2 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        dec.step()
        tok_host.copy_(dec.ids, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e2)
    status = runtime.device_status()
    times = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(times, op=torch.distributed.ReduceOp.MAX)
    ms, e2e_ms = times.tolist()
    dec.release()
    # Every rank runs the profiled step: it holds the same collectives as a step.
    breakdown = dec.profile_step() if args.breakdown else None
    dec_ar_mode = dec.ar.mode if dec.ar is not None else None
    fused = fused and dec_ar_mode is not None
    if status != 0:
        raise RuntimeError(f"device error word {status} after the timed region")

    # Bytes one step reads on this rank: every linear weight once, every KV page of
    # the context once (plus the new token's pages); x/y and norms are negligible.
    lin_host = sum(p.numel() * p.element_size() for m in dec.modules() for p in m.parameters(recurse=False)
                   if p.device.type == "cpu")
    lin_dev = sum(p.numel() * p.element_size() for l in dec.layers for p in l.parameters() if p.device.type == "cuda")
    lin_dev += sum(p.numel() * p.element_size() for p in dec.lm_head.parameters() if p.device.type == "cuda")
    kv_host, kv_dev = dec.kv_bytes()
    fill = min(1.0, (ctx + 1) / max_ctx)
    host_step, dev_step = lin_host + kv_host * fill, lin_dev + kv_dev * fill
    roof_ms = max(dev_step / (hbm_gbs * 1e9), host_step / (host_gbs * 1e9)) * 1e3
    # Whole-job figures: the slowest rank's lower bound, summed bytes, the
    # lowest host link.
    agg = torch.tensor([roof_ms, host_step, dev_step, -host_gbs], dtype=torch.float64, device="cuda")
    if world > 1:
        mx = agg[[0, 3]].clone()
        sm = agg[[1, 2]].clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(sm)
        roof_ms, host_gbs = mx[0].item(), -mx[1].item()
        host_step, dev_step = sm[0].item() / world, sm[1].item() / world
    step_ms = ms / K
    launches_per_step = dec.kernel_launches_per_step()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_llama70b(B, ctx, shape.layers)
    return {
        "metric": "decode tokens/s (Llama-3-70B arch, tensor parallel, weights and KV offloaded)",
        "value": round(B * K / (ms * 1e-3), 3), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(step_ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate / softmax)",
        "data": "synthetic: random N(0,0.02) weights, N(0,1) KV for the context, random token ids",
        "config": {"workload": f"BASELINE config 5: Llama-3-70B arch, {shape.layers} layers, batch {B}, ctx {ctx}, "
                               f"TP{world}, per-GPU HBM budget {budget_gb:g} GB"
                               + ("" if args.host_fraction is None else f", fixed host fraction {frac:g}"),
                   "host_fraction": round(frac, 4), "per_rank_host_fractions": [round(f, 4) for f in fracs],
                   "rank0_host_bytes": int(lin_host + kv_host),
                   "rank0_device_bytes": int(lin_dev + kv_dev), "build_s": round(build_s, 1),
                   "parallelism": f"tp{world}" if emulated == 1 else
                                  f"one rank of tp{emulated} on 1 GPU (its kernels and shapes, no all-reduce)",
                   "allreduce": "fused: row-parallel kernels publish, the next RMSNorm reduces over NVSwitch "
                                "multicast" if fused else "NCCL",
                   "allreduce_choice_ms": dec.allreduce_times_ms,
                   "l2": "tens of GB read per step exceed L2",
                   "timing": "CUDA events around K graph replays, max over ranks"},
        "roofline": {"bound": "hbm", "achieved": round((host_step + dev_step) / (step_ms * 1e-3) / 1e9, 2),
                     "peak": round((host_step + dev_step) / (roof_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "frac": round(roof_ms / step_ms, 4),
                     "traffic": round(dev_step * DRAM_PER_DEVICE_BYTE),
                     "traffic_basis": "per rank per step: device-resident weight and KV bytes x the DRAM/device-byte "
                                      "ratio of the linear captures",
                     "peak_model": "slowest rank's max(device bytes / HBM, host bytes / its host link) per step; "
                                   "achieved and peak are per-rank averages of the bytes",
                     "hbm_gbs": hbm_gbs, "hbm_peak_kind": peak_kind, "host_link_gbs_min": round(host_gbs, 2)},
        "e2e": {"value": round(B * K / (e2e_ms * 1e-3), 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 8 * B},
        "gpu_launches": launches_per_step * K, "clocks": clocks.summary(),
        **({"cpu_baseline": cpu} if cpu is not None else {}),
        **({"breakdown_ms": breakdown,
            "breakdown_basis": "rank 0, one eager step outside the timed region, CUDA events around each op group "
                               "(kernels serialized by the events)"} if breakdown is not None else {}),
    }


def rank_shape(shape, tp: int):
    """The per-rank layer shapes of a TP-``tp`` decoder as a one-rank model:
    query heads, KV heads and FFN features divided by ``tp``, lm_head rows as one
    rank's vocabulary shard.  The hidden size, head size and depth stay."""
    import dataclasses

    from directaccesskernel_b200.llama_tp import vocab_rows_per_rank

    if shape.heads % tp or shape.kv_heads % tp or shape.ffn % tp:
        raise ValueError(f"heads {shape.heads}, kv_heads {shape.kv_heads} and ffn {shape.ffn} must divide by {tp}")
    return dataclasses.replace(shape, heads=shape.heads // tp, kv_heads=shape.kv_heads // tp, ffn=shape.ffn // tp,
                               vocab=vocab_rows_per_rank(shape.vocab, tp))


def balanced_host_fractions(mean_frac: float, bandwidths: list[float], lo: float = 0.0) -> list[float]:
    """Per-rank host fractions whose mean is ``mean_frac`` and which are proportional
    to the ranks' host bandwidths, clamped to [lo, 1] (lo keeps the device part
    within the HBM budget); clamped ranks hand their excess to the others."""
    n = len(bandwidths)
    fr = [mean_frac] * n
    free = list(range(n))
    total = mean_frac * n
    for _ in range(n):
        bw = sum(bandwidths[i] for i in free)
        fixed = sum(fr[i] for i in range(n) if i not in free)
        for i in free:
            fr[i] = (total - fixed) * bandwidths[i] / bw
        out = [i for i in free if fr[i] > 1.0 or fr[i] < lo]
        if not out:
            break
        for i in out:
            fr[i] = min(1.0, max(lo, fr[i]))
            free.remove(i)
        if not free:
            break
    return fr


def cpu_baseline_llama70b(batch: int = 32, ctx: int = 16384, layers: int = 80):
    """The oracle port on the host cores for one config-5 decode step: numpy FP32
    of one Llama-3-70B layer's linears at batch 32 and of one sequence's GQA
    attention over its 16384-token context, extrapolated to 32 sequences and 80
    layers (the CPU cannot hold the model; labelled extrapolated)."""
    import numpy as np

    import oracle
    import oracle.attention as oatt

    h, f, hq, hkv, d = 8192, 28672, 64, 8, 128
    rng = np.random.default_rng(0)
    shapes = [(hq * d, h), (hkv * d, h), (hkv * d, h), (h, hq * d), (f, h), (f, h), (h, f)]
    t_lin = 0.0
    for shp in shapes:
        w = rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
        x = rng.standard_normal((batch, shp[1]), dtype=np.float32)
        t = time.perf_counter()
        oracle.linear(x, w, acc=np.float32)
        t_lin += time.perf_counter() - t
        del w
    k = rng.standard_normal((1, hkv, ctx, d), dtype=np.float32)
    v = rng.standard_normal((1, hkv, ctx, d), dtype=np.float32)
    q = rng.standard_normal((1, hq, 1, d), dtype=np.float32)
    t = time.perf_counter()
    oatt.decode_attention_grouped(q, k, v, 1.0 / math.sqrt(d))
    t_att = time.perf_counter() - t
    t_step = layers * (t_lin + batch * t_att)
    return {"value": round(batch / t_step, 5), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"one Llama-3-70B layer's 7 linears at batch {batch} + one sequence's attention over "
                      f"{ctx} tokens (numpy FP32), extrapolated to {batch} sequences x {layers} layers (extrapolated)"}


def cpu_baseline_opt66b(reps: int = 2):
    """The oracle port on the host cores: numpy FP32 x @ W^T of one OPT-66B decoder
    layer's six linears at batch 1, extrapolated to the whole model by parameter
    count (the CPU cannot hold the 263 GB FP32 model)."""
    import numpy as np

    import oracle

    h, f = 9216, 36864
    rng = np.random.default_rng(0)
    shapes = [(h, h)] * 4 + [(f, h), (h, f)]
    ws = [rng.standard_normal(s, dtype=np.float32) * np.float32(0.02) for s in shapes]
    layer_params = sum(a * b for a, b in shapes)
    best = float("inf")
    for _ in range(reps):
        x = rng.standard_normal((1, h), dtype=np.float32)
        t = time.perf_counter()
        for w in ws:
            y = oracle.linear(x if w.shape[1] == h else np.zeros((1, f), np.float32), w, acc=np.float32)
        best = min(best, time.perf_counter() - t)
        del y
    total_params = 65_719_701_504
    t_token = best * total_params / layer_params
    return {"value": round(1.0 / t_token, 5), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": "one OPT-66B decoder layer (6 linears, 1.02 B params, numpy FP32, batch 1), best of "
                      f"{reps}, extrapolated to 65.7 B params (extrapolated)"}


def run_reference(args):
    """Reference arm: the reference's computation of the path on the host cores
    (the oracle port: numpy FP32, all threads), on this arm's metric and config."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    if args.workload in ("attention", "opt66b", "llama70b"):
        fn = {"attention": cpu_baseline_attention, "opt66b": cpu_baseline_opt66b,
              "llama70b": lambda: cpu_baseline_llama70b(args.batch, args.ctx, args.layers)}[args.workload]
        metric, unit = {
            "attention": ("split-KV decode attention KV GB/s", "GB/s"),
            "opt66b": ("decode tokens/s (OPT-66B arch, HBM weight budget)", "tokens/s"),
            "llama70b": ("decode tokens/s (Llama-3-70B arch, tensor parallel, weights and KV offloaded)", "tokens/s"),
        }[args.workload]
        for _ in range(max(0, min(args.warmup, 1))):
            fn(budget_s=2.0) if args.workload == "attention" else fn()
        t0 = time.perf_counter()
        runs = [fn() for _ in range(args.steps)]
        elapsed = time.perf_counter() - t0
        v = statistics.median(r["value"] for r in runs)
        cpu = dict(runs[0], value=v)
        return {
            "metric": metric, "impl": "reference", "value": v, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(elapsed / max(1, args.steps) * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": "BASELINE " + {"attention": "config 3", "opt66b": "config 4",
                                                  "llama70b": "config 5"}[args.workload] + " sample on host cores"},
            "cpu_baseline": cpu,
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    prefill, tokens, ratios = linear_sweep(args)
    metric, config = linear_metric_config(prefill, tokens, ratios, args.gpus)
    sweep = CpuLinearSweep(tokens, ratios, "torch")
    t0 = time.perf_counter()
    times = sweep.timed_passes(args.steps, warmup=args.warmup)
    elapsed = time.perf_counter() - t0
    # The median pass, as the GPU arm's cpu_baseline reports it.
    v = round(sweep.bytes_per_pass / statistics.median(times) / 1e9, 3)
    sample, threads = sweep.sample(), sweep.threads
    del sweep
    port = CpuLinearSweep(tokens, ratios, "port")
    pt = port.timed_passes(max(1, min(args.steps, 3)), warmup=1)
    port_v = round(port.bytes_per_pass * len(pt) / sum(pt) / 1e9, 3)
    del port
    return {
        "metric": metric, "impl": "reference",
        "value": v, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sum(times) / len(times) * 1e3, 2), "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 else "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic N(0,0.02) weights, N(0,1) activations",
        "config": config,
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": sample + f"; median of {len(times)} timed steps, one pass per step",
                         "port_value": port_v, "port_kind": "port (numpy oracle, same passes)"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(elapsed, 2),
    }


def main():
    args = parse_args()
    if args.impl == "reference":
        line = run_reference(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        # NCCL reports each communicator's set-up (rank, nranks, Init COMPLETE)
        # on stderr, unless the caller chose its own NCCL logging.
        if "NCCL_DEBUG" not in os.environ:
            os.environ.update(NCCL_DEBUG="INFO", NCCL_DEBUG_SUBSYS="INIT", NCCL_DEBUG_FILE="/dev/stderr")
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        probe = torch.ones(1, device="cuda")
        torch.distributed.all_reduce(probe)
        torch.cuda.synchronize()
        print(f"[bench] rank {rank}: NCCL {'.'.join(map(str, torch.cuda.nccl.version()))} communicator up, "
              f"nranks={torch.distributed.get_world_size()}, all-reduce check {int(probe.item())} == {world}",
              file=sys.stderr, flush=True)
    try:
        fn = {"attention": run_attention, "opt66b": run_opt66b, "llama70b": run_llama70b,
              "plan-sweep": run_plan_sweep, "read-ceiling": run_read_ceiling}.get(args.workload, run_linear)
        line = fn(args, torch, rank, world)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
