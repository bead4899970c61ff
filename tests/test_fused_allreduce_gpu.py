"""Row-parallel linear with its all-reduce fused into the tcgen05 kernel
(dak_linear_split_allreduce) against the unfused path: per-rank linear plus an
NCCL all-reduce.  Runs with as many ranks as the box has GPUs (1 or 2 here),
over several consecutive calls (epochs and buffer parities) and CUDA-graph
replays, with weights split between pinned host memory and HBM."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max())


def _worker(rank, world, port, q, multicast, dtype=torch.float16):
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from directaccesskernel_b200 import runtime
        from directaccesskernel_b200.tp import SymmetricAllReduce

        errs = []
        N, Kr = 4096, 1024
        ar = SymmetricAllReduce(slot_elems=64 * N, multicast=multicast, dtype=dtype)
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        w = (torch.randn(Kr, N, generator=g, device="cuda") * 0.02).to(dtype)  # this rank's [K_r, N] shard
        w_host = w[:, :1024].contiguous().cpu().pin_memory()
        w_dev = w[:, 1024:].contiguous()
        for ntok in (1, 32, 64, 32, 5):
            x = torch.randn(ntok, Kr, generator=g, device="cuda").to(dtype)
            y = torch.empty(ntok, N, dtype=dtype, device="cuda")
            runtime.linear_split(x, y, w_host, w_dev, allreduce=ar)
            ref = (x.float() @ w.float()).contiguous()
            dist.all_reduce(ref)
            errs.append(_rel(y, ref))
        # CUDA graph: three fused calls captured, replayed twice with new inputs.
        xs = [torch.randn(32, Kr, generator=g, device="cuda").to(dtype) for _ in range(3)]
        ys = [torch.empty(32, N, dtype=dtype, device="cuda") for _ in range(3)]
        for i in range(3):
            runtime.linear_split(xs[i], ys[i], w_host, w_dev, allreduce=ar)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(3):
                runtime.linear_split(xs[i], ys[i], w_host, w_dev, allreduce=ar)
        for _ in range(2):
            for i in range(3):
                xs[i].copy_(torch.randn(32, Kr, generator=g, device="cuda").to(dtype))
            graph.replay()
            torch.cuda.synchronize()
            for i in range(3):
                ref = (xs[i].float() @ w.float()).contiguous()
                dist.all_reduce(ref)
                errs.append(_rel(ys[i], ref))
        del graph
        q.put((rank, max(errs), runtime.device_status(), ar.mode))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), -1, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("multicast", [False, True])
@pytest.mark.parametrize("world", [1, 2])
def test_fused_allreduce_matches_nccl(world, multicast, dtype):
    """Peer-store mode, and the multimem mode where the box offers multicast
    (the context falls back to peer stores otherwise; the mode is reported)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, multicast, dtype)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, err, st, mode = q.get(timeout=600)
        res[r] = (err, st, mode)
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        err, st, mode = res[r]
        assert isinstance(err, float) and err <= 1e-2 and st == 0, res
        if not multicast:
            assert mode == "peer"
    print("fused all-reduce modes:", {r: res[r][2] for r in res})


def _consumer_worker(rank, world, port, q, N=4096):
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from directaccesskernel_b200 import runtime
        from directaccesskernel_b200.tp import SymmetricAllReduce

        Kr = 1024
        ar = SymmetricAllReduce(slot_elems=64 * N, consumer_reduces=True)
        if not ar.publish_only:
            q.put((rank, "no multicast", 0, ar.mode))
            return
        g = torch.Generator(device="cuda").manual_seed(200 + rank)
        gs = torch.Generator(device="cuda").manual_seed(7)  # same residual and weight on every rank
        w = (torch.randn(Kr, N, generator=g, device="cuda") * 0.02).half()
        w_host, w_dev = w[:, :512].contiguous().cpu().pin_memory(), w[:, 512:].contiguous()
        errs = []
        for ntok in (1, 32, 5, 32):
            x = torch.randn(ntok, Kr, generator=g, device="cuda").half()
            res = torch.randn(ntok, N, generator=gs, device="cuda").half()
            wn = (1 + 0.1 * torch.randn(N, generator=gs, device="cuda")).half()
            y = torch.empty(ntok, N, dtype=torch.float16, device="cuda")  # layout only: not written
            runtime.linear_split(x, y, w_host, w_dev, allreduce=ar)
            state, out = res.clone(), torch.empty_like(res)
            ar.rmsnorm(y, state, wn, 1e-5, out)
            ref = (x.float() @ w.float()).contiguous()
            dist.all_reduce(ref)
            h = ref.half() + res
            hf = h.float()
            out_ref = wn * (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5)).half()
            errs += [_rel(state, h), _rel(out, out_ref)]
        q.put((rank, max(errs), runtime.device_status(), ar.mode))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), -1, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("N", [4096, 4104])
def test_consumer_side_reduction_in_rmsnorm(N):
    """Publish-only linear + dak_rmsnorm_allreduce against linear + NCCL all-reduce
    + residual add + RMSNorm; needs 2 GPUs with NVSwitch multicast.  4096
    columns take the 16-byte multicast reads, 4104 the single-column ones."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_consumer_worker, args=(r, 2, port, q, N)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, err, st, mode = q.get(timeout=600)
        res[r] = (err, st, mode)
    for p in procs:
        p.join(timeout=120)
    if all(v[0] == "no multicast" for v in res.values()):
        pytest.skip("no NVSwitch multicast on this box")
    for r in range(2):
        err, st, mode = res[r]
        assert isinstance(err, float) and err <= 1e-2 and st == 0, res
