"""GPU parity at the benchmark configurations, against the CPU oracle.

The shapes are the configurations the reference benchmarks name (Llama-3-8B
d=4096, ff=14336 at ratios 0.4/0.6/0.8/0.9; Llama-3-70B d=8192, ff=28672 at
ratio 0.8), run through the same entry points as the rest of the suite:
full outputs wherever the fp32 oracle finishes in seconds, sampled rows
(every 256-row tile boundary included) beyond that.  Inputs are seeded bf16
draws with the benchmark distributions (x ~ N(0,1), u ~ N(0,1/in),
v ~ N(0,1/r)); the oracle sees exactly the device's bf16 values.

Tolerance (the north-star criterion): relative Frobenius error <= 5e-3 and
max-abs error <= 2e-2 x RMS(reference) against fp32.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import svdmlp_oracle as orc
from helpers import assert_close, to_dev, to_np

pytestmark = pytest.mark.gpu

D8, FF8 = 4096, 14336
D70, FF70 = 8192, 28672


def _factors(d, ff, r, seed, dev):
    """bf16 device factors (u ~ N(0,1/in), v ~ N(0,1/r)) and their fp32 host copies."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def mat(rows, cols):
        return (torch.randn(rows, cols, generator=g, device=dev) / math.sqrt(rows)).to(torch.bfloat16)

    dev_f = [mat(d, r), mat(r, ff), mat(d, r), mat(r, ff), mat(ff, r), mat(r, d)]
    return dev_f, [to_np(t) for t in dev_f]


def _x(m, d, seed, dev):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    xd = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
    return xd, to_np(xd)


def _sample_rows(m, extra=64, seed=0):
    """First and last row of every 256-row tile, plus `extra` random rows."""
    rows = {0, m - 1}
    for t in range(0, m, 256):
        rows.update((t, min(t + 255, m - 1)))
    rows.update(np.random.default_rng(seed).integers(0, m, extra).tolist())
    return np.array(sorted(rows))


@pytest.fixture(scope="module")
def ops_mod():
    from svdflash_b200.kernels import ops
    return ops


# ------------------------------------------------------------- config 1
def test_config1_full_output(cuda_device, ops_mod):
    """Config 1 (8B layer, ratio 0.9 -> r = 2867, 1024 tokens): all rows."""
    r = orc.benchmark_rank(D8, FF8, 0.9)
    fd, fh = _factors(D8, FF8, r, 11, cuda_device)
    xd, xh = _x(1024, D8, 12, cuda_device)
    layer = ops_mod.pack_svd_layer(*fd)
    y = ops_mod.svd_mlp_packed(layer, xd)
    ops_mod.check_device_status(cuda_device)
    assert_close(to_np(y), orc.svd_mlp(xh, *fh), what="config 1, all 1024 rows")


# ---------------------------------------------- configs 2 and 5: ranks x tokens
@pytest.mark.parametrize("ratio", [0.4, 0.6, 0.8])
def test_8b_ranks_decode_and_prefill(cuda_device, ops_mod, ratio):
    """r = 1274 / 1911 / 2548 at 8, 32 and 128 tokens (the whole-layer and
    per-stage decode kernels) and at 1024 tokens (CTA-pair kernels)."""
    r = orc.benchmark_rank(D8, FF8, ratio)
    assert r == {0.4: 1274, 0.6: 1911, 0.8: 2548}[ratio]
    fd, fh = _factors(D8, FF8, r, 20 + int(ratio * 10), cuda_device)
    layer = ops_mod.pack_svd_layer(*fd)
    for m in (8, 32, 128, 1024):
        xd, xh = _x(m, D8, 100 + m, cuda_device)
        y = ops_mod.svd_mlp_packed(layer, xd)
        ops_mod.check_device_status(cuda_device)
        assert_close(to_np(y), orc.svd_mlp(xh, *fh), what=f"8B r={r} M={m}")


def test_8b_decode_ranks_at_ratio_09(cuda_device, ops_mod):
    """Config 2 at r = 2867 for 1, 8, 32 and 128 tokens, full outputs."""
    r = orc.benchmark_rank(D8, FF8, 0.9)
    fd, fh = _factors(D8, FF8, r, 30, cuda_device)
    layer = ops_mod.pack_svd_layer(*fd)
    for m in (1, 8, 32, 128):
        xd, xh = _x(m, D8, 200 + m, cuda_device)
        y = ops_mod.svd_mlp_packed(layer, xd)
        ops_mod.check_device_status(cuda_device)
        assert_close(to_np(y), orc.svd_mlp(xh, *fh), what=f"8B decode M={m}")


@pytest.mark.parametrize("m", [2048, 8192, 32768])
def test_8b_batch4_sampled_rows(cuda_device, ops_mod, m):
    """Config 5 at batch 4 (4 x 512, 4 x 2048, 4 x 8192 tokens), ratio 0.9:
    sampled rows against the oracle, and every row finite."""
    r = orc.benchmark_rank(D8, FF8, 0.9)
    fd, fh = _factors(D8, FF8, r, 40, cuda_device)
    xd, xh = _x(m, D8, 41, cuda_device)
    layer = ops_mod.pack_svd_layer(*fd)
    y = ops_mod.svd_mlp_packed(layer, xd)
    ops_mod.check_device_status(cuda_device)
    assert bool(torch.isfinite(y.float()).all())
    rows = _sample_rows(m, extra=64 if m <= 8192 else 32)
    assert_close(to_np(y)[rows], orc.svd_mlp(xh[rows], *fh), what=f"8B batch-4 M={m} sampled")


# ------------------------------------------------------------- config 4
@pytest.fixture(scope="module")
def layer70(cuda_device):
    r = orc.benchmark_rank(D70, FF70, 0.8)
    assert r == 5097
    fd, fh = _factors(D70, FF70, r, 70, cuda_device)
    xd, xh = _x(256, D70, 71, cuda_device)
    return r, fd, fh, xd, xh


def test_70b_layer_full_output(cuda_device, ops_mod, layer70):
    """Config 4 shape (d = 8192, ff = 28672, r = 5097) at 256 tokens, all rows."""
    r, fd, fh, xd, xh = layer70
    layer = ops_mod.pack_svd_layer(*fd)
    y = ops_mod.svd_mlp_packed(layer, xd)
    ops_mod.check_device_status(cuda_device)
    ref = orc.svd_mlp(xh, *fh)
    assert_close(to_np(y), ref, what="70B layer, 256 tokens")
    # the same layer at decode sizes (per-stage and whole-layer kernels)
    for m in (1, 64):
        ym = ops_mod.svd_mlp_packed(layer, xd[:m])
        assert_close(to_np(ym), ref[:m], what=f"70B layer, {m} tokens")
    ops_mod.check_device_status(cuda_device)


@pytest.mark.parametrize("world", [2, 8])
def test_70b_tensor_parallel_shards_on_one_gpu(cuda_device, ops_mod, layer70, world):
    """The ff-sharded 70B layer, `world` ranks emulated on one GPU: each
    rank's fp16 [M, r] partial, summed rank after rank in fp16 (what an
    ncclHalf all-reduce rounds), then . v_down: the full layer."""
    from svdflash_b200.tp import TensorParallelSvdMlp
    r, fd, fh, xd, xh = layer70
    total = None
    for p in range(world):
        sh = TensorParallelSvdMlp(*fd, rank=p, world=world, reduce_dtype=torch.float16, mode="allreduce")
        buf = sh._partial_buffer(xd.shape[0], cuda_device).clone()
        ops_mod.forward_partial_packed(sh.layer, xd, buf[:, :r])
        total = buf if total is None else total + buf
        if p < world - 1:
            del sh
    y = ops_mod.down_finish_packed(sh.layer, total[:, :r])
    ops_mod.check_device_status(cuda_device)
    assert_close(to_np(y), orc.svd_mlp(xh, *fh), what=f"70B TP {world} shards")


# ------------------------------------------- building blocks through the ABI
@pytest.mark.parametrize("m,n,k", [(1, 129, 131), (17, 1000, 777), (129, 257, 1025), (300, 513, 64),
                                   (1024, 4096, 2867), (2048, 2867, 4096)])
def test_dense_matmul_odd_shapes(cuda_device, ops_mod, m, n, k):
    """pallas_ops.dense_matmul -> svdmlp_gemm (the plain tcgen05 GEMM that
    replaces nki_matmul_fully_optimized_), decode and CTA-pair plans."""
    rng = np.random.default_rng(m + n + k)
    a = orc.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
    w = orc.bf16_round(rng.standard_normal((k, n), dtype=np.float32) / np.float32(np.sqrt(k)))
    c = ops_mod.dense_matmul(to_dev(a, cuda_device), to_dev(w, cuda_device))
    assert tuple(c.shape) == (m, n) and c.dtype == torch.bfloat16
    # one bf16 rounding of the output: 2^-8 relative per element
    ref = a @ w
    assert_close(to_np(c), ref, rel=5e-3, max_abs_rms=2e-2, what=f"gemm {m}x{n}x{k}")


@pytest.mark.parametrize("m,ff,r,d", [(8, 1024, 300, 512), (200, 2048, 520, 1024), (1024, 14336, 2867, 4096)])
def test_down_partial_fp32(cuda_device, ops_mod, m, ff, r, d):
    """svdmlp_down_partial: the fp32 [M, r] partial h . u_down of the
    tensor-parallel exchange, from a caller's bf16 H."""
    x, f = orc.make_inputs(300 + m, m, d, ff, r)
    hb = orc.bf16_round(orc.fused_gate_up(x, *f[:4]))
    layer = ops_mod.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    part = ops_mod.down_partial_packed(layer, to_dev(hb, cuda_device))
    ops_mod.check_device_status(cuda_device)
    assert part.dtype == torch.float32 and tuple(part.shape) == (m, r)
    # H is converted to fp16 on the device (one rounding), the sum is fp32
    assert_close(to_np(part), hb @ f[4], what=f"down_partial {m}x{ff}x{r}")
