"""fp16 range of the intermediates, on the GPU.

The layer keeps X.u, H = SiLU(g) * u and H.u_down in fp16 (with fp32
accumulation).  Moderate activation outliers stay inside fp16's range and
must match the fp32 oracle at the usual tolerance; outliers large enough to
push H past 65504 must be reported (SvdMlpRangeError from
check_device_status), never returned silently; weights that fp16 cannot
hold are refused when they are packed."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import svdmlp_oracle as orc
from helpers import assert_close, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from svdflash_b200.kernels import ops as o
    return o


def _layer(ops, dev, seed, m, d, ff, r, col_scale=None):
    x, f = orc.make_inputs(seed, m, d, ff, r)
    f = list(f)
    if col_scale is not None:
        # one rank component of the gate carried by large factor entries:
        # u_gate column j times s and v_gate row j times 1/s leave the product
        # unchanged but make X.u_gate large in that column
        j, s = col_scale
        f[0] = f[0].copy()
        f[1] = f[1].copy()
        f[0][:, j] = orc.bf16_round(f[0][:, j] * np.float32(s))
        f[1][j, :] = orc.bf16_round(f[1][j, :] / np.float32(s))
    layer = ops.pack_svd_layer(*[to_dev(a, dev) for a in f])
    return x, f, layer


@pytest.mark.parametrize("m", [4, 40, 300])  # whole-layer decode, per-stage decode, CTA pairs
def test_moderate_row_outliers_match_the_oracle(cuda_device, ops, m):
    """A few rows 16x the typical scale (their H up to ~256x).  The layer is
    independent per row, so the criterion is applied per row (each row
    against its own RMS): against the RMS of the whole output, which the
    outlier rows dominate, even one bf16 rounding of an outlier row's output
    exceeds 2e-2 x RMS."""
    x, f, layer = _layer(ops, cuda_device, 500 + m, m, 1024, 2048, 300)
    x = x.copy()
    x[:: max(1, m // 4)] *= 16.0
    x = orc.bf16_round(x)
    y = to_np(ops.svd_mlp_packed(layer, to_dev(x, cuda_device)))
    ops.check_device_status(cuda_device)
    ref = orc.svd_mlp(x, *f)
    assert orc.error_metrics(y, ref)["rel_fro"] <= 5e-3
    for i in range(m):
        assert_close(y[i], ref[i], what=f"16x row outliers, M={m}, row {i}")


@pytest.mark.parametrize("m", [4, 40, 300])
def test_large_row_outliers_are_reported(cuda_device, ops, m):
    from svdflash_b200 import _lib
    x0, f, layer = _layer(ops, cuda_device, 600 + m, m, 1024, 2048, 300)
    x = x0.copy()
    x[m // 2] *= 1000.0  # one row 1000x: SiLU(g) * u reaches ~1e6 there, past fp16
    x = orc.bf16_round(x)
    assert np.abs(orc.fused_gate_up(x, *f[:4])).max() > 65504.0
    ops.check_device_status(cuda_device)  # nothing pending before the call
    ops.svd_mlp_packed(layer, to_dev(x, cuda_device))
    with pytest.raises(_lib.SvdMlpRangeError):
        ops.check_device_status(cuda_device)
    # reported once, then cleared: an in-range call afterwards is clean
    y2 = ops.svd_mlp_packed(layer, to_dev(x0, cuda_device))
    ops.check_device_status(cuda_device)
    assert_close(to_np(y2), orc.svd_mlp(x0, *f), what=f"after a reported range error, M={m}")


def test_large_factor_columns(cuda_device, ops):
    """A rank component carried by factor entries 64x the usual size stays
    within fp16 and matches; one carried by entries 2^14 x larger pushes
    X.u_gate past fp16 and is reported."""
    from svdflash_b200 import _lib
    m = 200
    x, f, layer = _layer(ops, cuda_device, 700, m, 1024, 2048, 300, col_scale=(5, 64.0))
    y = ops.svd_mlp_packed(layer, to_dev(x, cuda_device))
    ops.check_device_status(cuda_device)
    assert_close(to_np(y), orc.svd_mlp(x, *f), what="factor column x64")
    x, f, layer = _layer(ops, cuda_device, 701, m, 1024, 2048, 300, col_scale=(5, 2.0 ** 20))
    assert np.abs(x @ f[0]).max() > 65504.0
    ops.svd_mlp_packed(layer, to_dev(x, cuda_device))
    with pytest.raises(_lib.SvdMlpRangeError):
        ops.check_device_status(cuda_device)


def test_weights_beyond_fp16_are_refused_at_pack(cuda_device, ops):
    from svdflash_b200 import _lib
    _, f = orc.make_inputs(800, 1, 256, 512, 64)
    f = [a.copy() for a in f]
    f[1][3, 7] = 1.0e6   # v_gate is stored as fp16 (it multiplies the fp16 X.u)
    with pytest.raises(_lib.SvdMlpRangeError):
        ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    f[1][3, 7] = 6.0e4   # below the fp16 limit: accepted
    ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])


def test_bf16_h_beyond_fp16_is_reported_by_xuv(cuda_device, ops):
    """fused_xuv / xuv_matmul on a full layer converts the caller's bf16 H to
    fp16; an H entry fp16 cannot hold is reported."""
    from svdflash_b200 import _lib
    m, d, ff, r = 32, 512, 1024, 200
    x, f = orc.make_inputs(900, m, d, ff, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    h = orc.bf16_round(orc.fused_gate_up(x, *f[:4]))
    h[3, 5] = 2.0e5
    ops.check_device_status(cuda_device)
    ops.xuv_packed(layer, to_dev(h, cuda_device))
    with pytest.raises(_lib.SvdMlpRangeError):
        ops.check_device_status(cuda_device)
