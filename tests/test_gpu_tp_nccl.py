"""Tensor parallelism on two GPUs over NCCL (plain collectives, NVLS off):
TensorParallelSvdMlp.forward_rows in both modes against forward() on the whole
batch and against the oracle, with and without a residual and with `out=`.
Each rank is a child process with its own GPU; the test is skipped on a box
with fewer than two GPUs."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import svdmlp_oracle as orc
from helpers import assert_close

pytestmark = pytest.mark.gpu

M, D, FF, R = 256, 512, 1024, 200


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    out = {}
    try:
        from svdflash_b200.tp import TensorParallelSvdMlp
        x, f = orc.make_inputs(90, M, D, FF, R)
        res = orc.bf16_round(np.random.default_rng(91).standard_normal((M, D), dtype=np.float32))
        fd = [torch.from_numpy(a).to(dev, torch.bfloat16) for a in f]
        xd = torch.from_numpy(x).to(dev, torch.bfloat16)
        rd = torch.from_numpy(res).to(dev, torch.bfloat16)
        rows = M // world
        mine = slice(rank * rows, (rank + 1) * rows)
        for mode in ("allreduce", "split"):
            tp = TensorParallelSvdMlp(*fd, rank=rank, world=world, mode=mode, collectives="nccl")
            full = tp.forward(xd)
            full_res = tp.forward(xd, residual=rd)
            got = tp.forward_rows(xd[mine].contiguous())
            buf = torch.empty(rows, D, dtype=torch.bfloat16, device=dev)
            got_res = tp.forward_rows(xd[mine].contiguous(), residual=rd[mine].contiguous(), out=buf)
            torch.cuda.synchronize()
            out[mode] = {
                "full": full.float().cpu().numpy(), "full_res": full_res.float().cpu().numpy(),
                "rows": got.float().cpu().numpy(), "rows_res": got_res.float().cpu().numpy(),
                "out_is_buf": got_res.data_ptr() == buf.data_ptr(),
                "rows_equal_full": bool(torch.equal(got, full[mine])),
                "rows_res_equal_full": bool(torch.equal(got_res, full_res[mine])),
            }
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


def test_forward_rows_matches_forward_on_two_gpus(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    for r in range(world):
        assert isinstance(outs[r], dict), outs[r]
    x, f = orc.make_inputs(90, M, D, FF, R)
    res = orc.bf16_round(np.random.default_rng(91).standard_normal((M, D), dtype=np.float32))
    ref = orc.svd_mlp(x, *f)
    rows = M // world
    for mode in ("allreduce", "split"):
        for r in range(world):
            o = outs[r][mode]
            mine = slice(r * rows, (r + 1) * rows)
            assert_close(o["full"], ref, what=f"{mode} forward rank {r}")
            assert_close(o["full_res"], ref + res, what=f"{mode} forward+residual rank {r}")
            assert_close(o["rows"], ref[mine], what=f"{mode} forward_rows rank {r}")
            assert_close(o["rows_res"], (ref + res)[mine], what=f"{mode} forward_rows+residual rank {r}")
            assert o["out_is_buf"], f"{mode}: out= not honoured"
            assert o["rows_equal_full"] and o["rows_res_equal_full"], f"{mode}: rows differ from forward()"
        np.testing.assert_array_equal(outs[0][mode]["full"], outs[1][mode]["full"])
