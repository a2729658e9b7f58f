"""ff-sharded tensor parallelism: the partition and the all-reduce, on
world-size-2 gloo ranks on the CPU with the oracle's arithmetic; plus
failure detection on the host (a rank that never joins)."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import svdmlp_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        x, f = orc.make_inputs(21, 12, 64, 128, 40, 24)
        shard = orc.shard_factors(f, rank, world)
        part = torch.from_numpy(orc.shard_partial(x, shard))
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        y = orc.tp_finish(part.numpy(), f[5])
        q.put((rank, y))
    finally:
        dist.destroy_process_group()


def test_ff_sharded_layer_matches_single_rank():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, f = orc.make_inputs(21, 12, 64, 128, 40, 24)
    ref = orc.svd_mlp(x, *f)
    for r in range(world):
        np.testing.assert_allclose(outs[r], ref, rtol=1e-4, atol=1e-5)
    np.testing.assert_array_equal(outs[0], outs[1])


def _rows_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from svdflash_b200.tp import gather_rows_forward
        x, f = orc.make_inputs(23, 12, 64, 128, 40, 24)
        rows = x.shape[0] // world
        res = np.arange(x.size, dtype=np.float32).reshape(x.shape) / x.size

        def fwd(xx, residual=None):  # the whole layer, as every rank computes it
            y = orc.svd_mlp(xx.numpy(), *f)
            return torch.from_numpy(y + (0 if residual is None else residual.numpy()))

        mine = slice(rank * rows, (rank + 1) * rows)
        y = gather_rows_forward(fwd, torch.from_numpy(x[mine]), rank, world,
                                residual_rows=torch.from_numpy(res[mine]))
        q.put((rank, y.numpy()))
    finally:
        dist.destroy_process_group()


def test_row_sharded_io_gathers_and_returns_own_rows():
    """gather_rows_forward: each rank passes its row block of X and of the
    residual, the blocks are all-gathered, and each rank gets its own rows of
    the whole-batch result."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rows_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, f = orc.make_inputs(23, 12, 64, 128, 40, 24)
    res = np.arange(x.size, dtype=np.float32).reshape(x.shape) / x.size
    ref = orc.svd_mlp(x, *f) + res
    np.testing.assert_allclose(np.concatenate([outs[0], outs[1]]), ref, rtol=1e-6, atol=1e-6)


def test_shard_bounds_and_uneven_ff():
    from svdflash_b200.tp import shard_bounds
    assert [shard_bounds(14336, r, 8) for r in (0, 7)] == [(0, 1792), (12544, 14336)]
    with pytest.raises(ValueError):
        shard_bounds(100, 0, 3)
    with pytest.raises(ValueError):
        orc.shard_factors(orc.make_inputs(0, 2, 8, 10, 4)[1], 0, 3)


def _absent_peer_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        dist.destroy_process_group()   # leaves between steps, never joins the collective
        q.put((rank, "left"))
        return
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error:{type(e).__name__}"))


def test_rank_that_never_joins_times_out():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error:"), res
