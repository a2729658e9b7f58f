"""The library's collectives over NVLink peer memory (svdflash_b200.peer) and
the tensor-parallel layer that uses them, on two or more GPUs.

Each rank is a child process with its own GPU; skipped on a box with fewer
than two GPUs.  The collectives are checked bit for bit: the all-reduce and
the reduce-scatter against the fp32 sum in rank order rounded once to fp16
(computed here in NumPy), the all-gather against the inputs; with a ragged row
count, padded rows, repeated calls, and an fp16 overflow that must be
reported.  The layer (both modes, forward and forward_rows, eager and
captured in a CUDA graph) is checked against the oracle at the north-star
tolerance and must give the same bits on every rank; in the all-reduce mode
the exchange fused into the H.u_down GEMM must give the same bits as the
separate all-reduce kernel, at prefill, decode and ragged row counts."""
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


def _rank_matrix(seed, rank, m, c, scale=1.0):
    rng = np.random.default_rng(seed * 100 + rank)
    return (scale * rng.standard_normal((m, c))).astype(np.float16)


def _expected_sum(seed, world, m, c, scale=1.0):
    acc = np.zeros((m, c), dtype=np.float32)
    for p in range(world):
        acc += _rank_matrix(seed, p, m, c, scale).astype(np.float32)  # fp32, rank order
    with np.errstate(over="ignore"):
        return acc.astype(np.float16)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    out = {}
    try:
        from svdflash_b200 import _lib
        from svdflash_b200.peer import PeerBuffer, layout, peer_access_everywhere
        from svdflash_b200.tp import TensorParallelSvdMlp
        out["access"] = peer_access_everywhere()
        # ---- the collectives on their own: ragged rows, padded columns
        m, c, ld = 37, 24, 32
        signal = int(_lib.load().svdmlp_peer_signal_bytes())
        scratch = int(_lib.load().svdmlp_peer_scratch_bytes(world, m, c))
        (off_a, off_s, off_g), total = layout([m * ld * 2, scratch, m * 48 * 2], signal)
        pb = PeerBuffer(total, rank, world)
        a = pb.view(off_a, (m, ld), torch.float16)
        rows_per = -(-m // world)
        r0, r1 = min(m, rank * rows_per), min(m, (rank + 1) * rows_per)
        sums, scatters, gathers = [], [], []
        for it in range(4):
            a.zero_()
            a[:, :c] = torch.from_numpy(_rank_matrix(it, rank, m, c)).to(dev)
            pb.allreduce_f16(off_a, m, c, ld, off_s)
            sums.append(a[:, :c].cpu().numpy().view(np.uint16).copy())
            a[:, :c] = torch.from_numpy(_rank_matrix(10 + it, rank, m, c)).to(dev)
            t = torch.full((rows_per, c), float("nan"), dtype=torch.float16, device=dev)
            pb.reduce_scatter_f16(off_a, m, c, ld, off_s, t)
            scatters.append(t[:r1 - r0].cpu().numpy().view(np.uint16).copy())
            g = pb.view(off_g, (m, 48), torch.bfloat16)
            g.fill_(float("nan"))
            g[r0:r1, :40] = torch.from_numpy(_rank_matrix(20 + it, rank, m, 40)[r0:r1].astype(np.float32)).to(
                dev, torch.bfloat16)
            pb.allgather(off_g, m, 80, 96)
            gathers.append(g[:, :40].float().cpu().numpy())
        pb.check_status()
        out.update(sums=sums, scatters=scatters, gathers=gathers, r0=r0, r1=r1)
        # an fp16 overflow in the sum is reported, not silent
        a.zero_()
        a[:, :c] = 40000.0
        pb.allreduce_f16(off_a, m, c, ld, off_s)
        try:
            pb.check_status()
            out["range"] = "not reported"
        except FloatingPointError:
            out["range"] = "reported"
        pb.check_status()  # cleared by the read
        pb.close()
        # ---- the layer
        x, f = orc.make_inputs(190, M, D, FF, R)
        res = orc.bf16_round(np.random.default_rng(191).standard_normal((M, D), dtype=np.float32))
        fd = [torch.from_numpy(v).to(dev, torch.bfloat16) for v in f]
        xd = torch.from_numpy(x).to(dev, torch.bfloat16)
        rd = torch.from_numpy(res).to(dev, torch.bfloat16)
        rows = M // world
        mine = slice(rank * rows, (rank + 1) * rows)
        for mode in ("allreduce", "split"):
            tp = TensorParallelSvdMlp(*fd, rank=rank, world=world, mode=mode, collectives="peer")
            full = tp.forward(xd)
            full_res = tp.forward(xd, residual=rd)
            got = tp.forward_rows(xd[mine].contiguous())
            nccl = TensorParallelSvdMlp(*fd, rank=rank, world=world, mode=mode, collectives="nccl").forward(xd)
            # captured: the collectives are kernels like the GEMMs
            static_x = xd.clone()
            y_static = torch.empty_like(full)
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                tp.forward(static_x, out=y_static)
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                tp.forward(static_x, out=y_static)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize(dev)
            replay_equal = bool(torch.equal(y_static, full))
            del graph
            tp.check_peer_status()
            out[mode] = {"full": full.float().cpu().numpy(), "full_res": full_res.float().cpu().numpy(),
                         "rows": got.float().cpu().numpy(), "nccl": nccl.float().cpu().numpy(),
                         "replay_equal": replay_equal, "peer": tp.peer_collectives()}
            if mode == "allreduce":
                # the exchange fused into H.u_down against the separate
                # all-reduce kernel: prefill (CTA-pair GEMM), decode and ragged
                # row counts on the same slots, one after another
                unf = TensorParallelSvdMlp(*fd, rank=rank, world=world, mode=mode, collectives="peer",
                                           fused_exchange=False)
                if not tp.fused_exchange:  # larger groups: force the fused path for this comparison
                    tp.close()
                    tp = TensorParallelSvdMlp(*fd, rank=rank, world=world, mode=mode, collectives="peer",
                                              fused_exchange=True)
                pairs = []
                for m_call in (M, 4, 37, M, 1):
                    a = tp.forward(xd[:m_call])
                    b = unf.forward(xd[:m_call])
                    pairs.append((m_call, a.float().cpu().numpy(), b.float().cpu().numpy()))
                tp.check_peer_status()
                unf.check_peer_status()
                unf.close()
                out[mode]["fused_vs_unfused"] = pairs
            tp.close()
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


def _run(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    for r in range(world):
        assert isinstance(outs[r], dict), outs[r]
    return outs


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_collectives_and_layer(cuda_device, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    outs = _run(world)
    m, c = 37, 24
    for r in range(world):
        o = outs[r]
        assert o["access"], "peer access expected on this box"
        for it in range(4):
            want = _expected_sum(it, world, m, c).view(np.uint16)
            np.testing.assert_array_equal(o["sums"][it], want, err_msg=f"all-reduce rank {r} call {it}")
            want_rs = _expected_sum(10 + it, world, m, c).view(np.uint16)[o["r0"]:o["r1"]]
            np.testing.assert_array_equal(o["scatters"][it], want_rs, err_msg=f"reduce-scatter rank {r}")
            rows_per = -(-m // world)
            want_g = np.concatenate([_rank_matrix(20 + it, p, m, 40)[min(m, p * rows_per):min(m, (p + 1) * rows_per)]
                                     for p in range(world)]).astype(np.float32)
            np.testing.assert_array_equal(o["gathers"][it], orc.bf16_round(want_g), err_msg=f"all-gather rank {r}")
        assert o["range"] == "reported"
    x, f = orc.make_inputs(190, M, D, FF, R)
    res = orc.bf16_round(np.random.default_rng(191).standard_normal((M, D), dtype=np.float32))
    ref = orc.svd_mlp(x, *f)
    rows = M // world
    for mode in ("allreduce", "split"):
        for r in range(world):
            o = outs[r][mode]
            assert o["peer"]
            assert_close(o["full"], ref, what=f"{mode} peer forward rank {r}")
            assert_close(o["full_res"], ref + res, what=f"{mode} peer forward+residual rank {r}")
            assert_close(o["rows"], ref[r * rows:(r + 1) * rows], what=f"{mode} peer forward_rows rank {r}")
            # two approximations of the same sum (NCCL's fp16 ring rounds at every
            # hop): each is held to the oracle above; against each other, twice the bound
            assert_close(o["full"], o["nccl"], rel=1e-2, max_abs_rms=4e-2, what=f"{mode} peer vs NCCL rank {r}")
            assert o["replay_equal"], f"{mode}: graph replay differs from eager"
            np.testing.assert_array_equal(o["full"], outs[0][mode]["full"])
            for m_call, fused, unfused in o.get("fused_vs_unfused", []):
                # same partials, same rank-order fp32 sums rounded once: the same bits
                np.testing.assert_array_equal(fused, unfused, err_msg=f"fused exchange, {m_call} rows, rank {r}")
                assert_close(fused, ref[:m_call], what=f"fused exchange {m_call} rows rank {r}")
        if mode == "allreduce":
            assert outs[0][mode]["fused_vs_unfused"], "fused exchange not exercised"
