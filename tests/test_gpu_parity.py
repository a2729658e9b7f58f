"""GPU parity of the sm_100a kernels against the CPU oracle (through the C ABI).

Tolerance (the north-star criterion): relative Frobenius error <= 5e-3 and
max-abs error <= 2e-2 x RMS(reference) against the fp32 oracle, on identical
bf16-grid inputs.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import svdmlp_oracle as orc
from helpers import assert_close, assert_close_bf16_output, to_dev, to_np

pytestmark = pytest.mark.gpu

# (S, H, R, I): the reference's tail shapes plus small odd cases.
SHAPES = [
    (1, 129, 131, 137),
    (129, 257, 257, 513),
    (257, 513, 513, 1025),
    (3, 257, 1025, 513),
    (13, 64, 40, 96),
    (128, 256, 64, 384),
    (200, 1024, 300, 2048),
]


def _ops():
    from svdflash_b200.kernels import ops
    return ops


@pytest.mark.parametrize("shape", SHAPES)
def test_svd_mlp_matches_oracle(cuda_device, shape):
    s, h, r, i = shape
    x, f = orc.make_inputs(100 + s, s, h, i, r)
    ref = orc.svd_mlp(x, *f)
    got = _ops().svd_mlp(to_dev(x, cuda_device), *[to_dev(a, cuda_device) for a in f])
    torch.cuda.synchronize()
    assert got.dtype == torch.bfloat16 and tuple(got.shape) == (s, h)
    assert_close(to_np(got), ref, what=f"svd_mlp {shape}")


@pytest.mark.parametrize("shape", SHAPES[:4])
def test_gate_up_and_xuv_match_oracle(cuda_device, shape):
    s, h, r, i = shape
    x, f = orc.make_inputs(200 + s, s, h, i, r)
    ops = _ops()
    hid = ops.fused_gate_up(to_dev(x, cuda_device), *[to_dev(a, cuda_device) for a in f[:4]])
    assert tuple(hid.shape) == (s, i)
    assert_close_bf16_output(to_np(hid), orc.fused_gate_up(x, *f[:4]), what=f"gate_up {shape}")
    hb = orc.bf16_round(orc.fused_gate_up(x, *f[:4]))
    y = ops.xuv_matmul(to_dev(hb, cuda_device), to_dev(f[4], cuda_device), to_dev(f[5], cuda_device))
    assert_close(to_np(y), orc.fused_xuv(hb, f[4], f[5]), what=f"xuv {shape}")


@pytest.mark.parametrize("shape", [(3, 257, 0, 513), (129, 256, 0, 1024), (64, 1024, 0, 4096)])
def test_dense_mlp_matches_oracle(cuda_device, shape):
    s, h, _, i = shape
    rng = np.random.default_rng(7)
    x = orc.bf16_round(rng.standard_normal((s, h), dtype=np.float32))
    wg, wu, wd = orc.make_dense(8, h, i)
    got = _ops().dense_mlp(*[to_dev(a, cuda_device) for a in (x, wg, wu, wd)])
    assert_close(to_np(got), orc.dense_mlp(x, wg, wu, wd), what=f"dense {shape}")


def test_golden_fixtures_on_gpu(cuda_device):
    import json
    import pathlib
    gdir = pathlib.Path(__file__).resolve().parent / "golden"
    index = json.loads((gdir / "index.json").read_text())
    ops = _ops()
    for name, meta in index.items():
        if name == "low_rank_dim" or not meta["full"]:
            continue
        z = np.load(gdir / f"{name}.npz")
        ins = {k: orc.from_bf16_bits(z[k]) for k in ("x", "u_gate", "v_gate", "u_up", "v_up", "u_down", "v_down")}
        got = ops.svd_mlp(*[to_dev(ins[k], cuda_device) for k in
                            ("x", "u_gate", "v_gate", "u_up", "v_up", "u_down", "v_down")])
        assert_close(to_np(got), z["svd_mlp"], what=f"golden {name}")


def test_residual_epilogue(cuda_device):
    s, h, r, i = 200, 1024, 300, 2048
    x, f = orc.make_inputs(5, s, h, i, r)
    res = orc.bf16_round(np.random.default_rng(6).standard_normal((s, h), dtype=np.float32))
    ops = _ops()
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    got = ops.svd_mlp_packed(layer, to_dev(x, cuda_device), residual=to_dev(res, cuda_device))
    assert_close(to_np(got), res + orc.svd_mlp(x, *f), what="residual")


def test_split_k_and_determinism(cuda_device):
    """Forced split-K factors agree with the unsplit kernel, and repeated runs are bitwise identical."""
    from svdflash_b200 import _lib
    lib = _lib.load()
    s, h, r, i = 256, 1024, 520, 2048
    x, f = orc.make_inputs(9, s, h, i, r)
    ops = _ops()
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    xd = to_dev(x, cuda_device)
    ref = orc.svd_mlp(x, *f)
    outs = []
    try:
        for splits in (1, 2, 3, 5):
            for st in range(4):
                lib.svdmlp_set_split_override(st, splits)
            y1 = ops.svd_mlp_packed(layer, xd)
            y2 = ops.svd_mlp_packed(layer, xd)
            torch.cuda.synchronize()
            assert torch.equal(y1, y2), f"splits={splits}: runs differ"
            assert_close(to_np(y1), ref, what=f"splits={splits}")
            outs.append(y1)
    finally:
        for st in range(4):
            lib.svdmlp_set_split_override(st, 0)
    ops.check_device_status(cuda_device)


def test_full_size_config1_properties(cuda_device):
    """Config 1 (8B, M=1024, r=2867) against the oracle on a row sample."""
    m, d, ff = 1024, 4096, 14336
    r = orc.benchmark_rank(d, ff, 0.9)
    assert r == 2867
    x, f = orc.make_inputs(1234, m, d, ff, r)
    ops = _ops()
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    y = ops.svd_mlp_packed(layer, to_dev(x, cuda_device))
    torch.cuda.synchronize()
    rows = np.arange(0, m, 37)
    ref = orc.svd_mlp(x[rows], *f)
    assert_close(to_np(y)[rows], ref, what="config1 sampled rows")
    ops.check_device_status(cuda_device)


def test_device_wait_timeout_reports_error(cuda_device):
    """A bounded device wait that expires is reported, and the context stays usable."""
    from svdflash_b200 import _lib
    lib = _lib.load()
    ws = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    import ctypes
    s = ctypes.c_void_p(stream)
    assert lib.svdmlp_workspace_init(ws.data_ptr(), ws.numel(), s) == 0
    assert lib.svdmlp_debug_wait_timeout(ws.data_ptr(), ws.numel(), 2_000_000, s) == 0
    assert lib.svdmlp_check_device_status(ws.data_ptr(), ws.numel(), s) == _lib.ERR_DEVICE_TIMEOUT
    # re-armed and usable
    assert lib.svdmlp_check_device_status(ws.data_ptr(), ws.numel(), s) == 0
    assert float((torch.ones(4, device=cuda_device) * 2).sum()) == 8.0


def test_split_tail_matches_whole_tiles(cuda_device):
    """The CTA-pair split tail (the last, partial wave's tiles split over K):
    at a shape whose dual gate/up GEMM has one full wave plus a partial one,
    the layer with and without the tail matches the oracle, and repeated runs
    with the tail are bitwise identical."""
    from svdflash_b200 import _lib
    lib = _lib.load()
    s, h, r, i = 512, 1024, 2048, 10240
    x, f = orc.make_inputs(13, s, h, i, r)
    ops = _ops()
    out = (ctypes.c_int * 6)()
    assert lib.svdmlp_plan_info(1, s, i, r, out) == 0 and out[4] > out[0] * out[1]   # tail units present
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    xd = to_dev(x, cuda_device)
    ref = orc.svd_mlp(x, *f)
    try:
        lib.svdmlp_set_split_tail(0)
        y_whole = ops.svd_mlp_packed(layer, xd)
        lib.svdmlp_set_split_tail(1)
        y1 = ops.svd_mlp_packed(layer, xd)
        y2 = ops.svd_mlp_packed(layer, xd)
        torch.cuda.synchronize()
    finally:
        lib.svdmlp_set_split_tail(1)
    ops.check_device_status(cuda_device)
    assert torch.equal(y1, y2)
    assert_close(to_np(y_whole), ref, what="whole tiles")
    assert_close(to_np(y1), ref, what="split tail")
