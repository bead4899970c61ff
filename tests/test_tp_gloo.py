"""Tensor-parallel sharding and collectives with world_size 2, 4 and 8 on CPU (gloo).

The per-rank compute is a plain nn.Linear on the rank's shard, so these tests
pin the sharding arithmetic and the collective wiring of
directaccesskernel_b200.tp; the GPU kernels behind each shard are covered by
the -m gpu tests."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        _run(rank, world, q)
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@torch.no_grad()
def _run(rank, world, q):
    from directaccesskernel_b200.tp import ColumnParallelLinear, RowParallelLinear, shard_cols, shard_rows

    torch.manual_seed(0)
    w = torch.randn(96, 64, dtype=torch.float64)
    x = torch.randn(3, 64, dtype=torch.float64)
    ref = x @ w.T
    step = 96 // world

    def local(shard):
        lin = torch.nn.Linear(shard.shape[1], shard.shape[0], bias=False, dtype=torch.float64)
        with torch.no_grad():
            lin.weight.copy_(shard)
        return lin

    col = ColumnParallelLinear(local(shard_rows(w, rank, world)), 96)
    y_col = col(x)
    col_sharded = ColumnParallelLinear(local(shard_rows(w, rank, world)), 96, gather_output=False)(x)
    row = RowParallelLinear(local(shard_cols(w, rank, world)), 64)
    y_row = row(x)
    # An MLP-style pair: column-parallel (sharded output) feeding row-parallel.
    w2 = torch.randn(64, 96, dtype=torch.float64)
    up = ColumnParallelLinear(local(shard_rows(w, rank, world)), 96, gather_output=False)
    down = RowParallelLinear(local(shard_cols(w2, rank, world)), 96, input_is_parallel=True)
    y_mlp = down(up(x))
    q.put((rank, float((y_col - ref).abs().max()), float((y_row - ref).abs().max()),
           float((col_sharded - ref[:, rank * step:(rank + 1) * step]).abs().max()),
           float((y_mlp - (x @ w.T) @ w2.T).abs().max())))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_column_and_row_parallel_match_unsharded(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(len(r) == 5 for r in res), res
    for rank, e_col, e_row, e_shard, e_mlp in res:
        assert e_col < 1e-12 and e_row < 1e-12 and e_shard < 1e-12 and e_mlp < 1e-10, (rank, e_col, e_row)


def _dead_peer_worker(rank, world, port, q):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        # This rank leaves between steps, with no collective in flight.
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush the message before leaving
        os._exit(0)
    from directaccesskernel_b200.tp import RowParallelLinear

    lin = torch.nn.Linear(32, 8, bias=False)
    row = RowParallelLinear(lin, 64)
    try:
        with torch.no_grad():
            row(torch.randn(2, 64))
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__))


def test_tp_dead_peer_is_detected_by_the_collective_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0] != "no error"


def test_shard_helpers_reject_uneven_splits():
    from directaccesskernel_b200.tp import shard_cols, shard_rows

    with pytest.raises(ValueError):
        shard_rows(torch.zeros(10, 4), 0, 3)
    with pytest.raises(ValueError):
        shard_cols(torch.zeros(4, 10), 0, 4)
