"""GPU tests of the contracted layer (svdmlp_forward_contracted,
pallas_ops.contracted_svd_mlp): at decode sizes each SwiGLU tile of H stays
in shared memory and is multiplied by its slice of u_down in the same unit;
T = H . u_down is summed from per-tile fp32 partials in a fixed order.  It
must match the oracle, repeat bit for bit, and agree with the four-stage
schedule; above 16 tokens it is the two-operator path."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import svdmlp_oracle as orc
from helpers import assert_close, assert_close_bf16_output, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from svdflash_b200.kernels import ops as o
    return o


@pytest.mark.parametrize("shape", [(1, 4096, 2867, 14336), (5, 4096, 2867, 14336), (16, 4096, 1911, 14336),
                                   (3, 1024, 700, 3584), (7, 257, 131, 513)])
def test_contracted_decode_matches_oracle(cuda_device, ops, shape):
    m, h, r, i = shape
    x, f = orc.make_inputs(400 + m, m, h, i, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    xd = to_dev(x, cuda_device)
    res = orc.bf16_round(np.random.default_rng(m).standard_normal((m, h), dtype=np.float32))
    rd = to_dev(res, cuda_device)
    y1 = ops.contracted_mlp_packed(layer, xd)
    y2 = ops.contracted_mlp_packed(layer, xd)
    yr = ops.contracted_mlp_packed(layer, xd, residual=rd)
    y4 = ops.svd_mlp_packed(layer, xd)
    torch.cuda.synchronize()
    ops.check_device_status(cuda_device)
    ref = orc.svd_mlp(x, *f)
    assert_close(to_np(y1), ref, what=f"contracted {shape}")
    assert_close(to_np(yr), res + ref, what=f"contracted + residual {shape}")
    assert torch.equal(y1, y2), "repeated contracted calls differ"
    assert_close_bf16_output(to_np(y1), to_np(y4), what=f"contracted vs four stages {shape}")


def test_contracted_70b_rank_two_tmem_passes(cuda_device, ops):
    """r = 5097: 40 rank tiles of T, more than one pass of TMEM columns."""
    m, h, r, i = 2, 8192, 5097, 28672
    g = torch.Generator(device=cuda_device)
    g.manual_seed(5)
    mk = lambda a, b: (torch.randn(a, b, generator=g, device=cuda_device) / float(np.sqrt(a))).to(torch.bfloat16)  # noqa: E731
    fd = [mk(h, r), mk(r, i), mk(h, r), mk(r, i), mk(i, r), mk(r, h)]
    xd = torch.randn(m, h, generator=g, device=cuda_device).to(torch.bfloat16)
    layer = ops.pack_svd_layer(*fd)
    y = ops.contracted_mlp_packed(layer, xd)
    ops.check_device_status(cuda_device)
    ref = orc.svd_mlp(to_np(xd), *[to_np(t) for t in fd])
    assert_close(to_np(y), ref, what="contracted 70B")


def test_contracted_api_above_decode_sizes(cuda_device, ops):
    """Above 16 tokens contracted_svd_mlp runs the two-operator path: the same
    bits as svd_mlp."""
    m, h, r, i = 200, 1024, 300, 2048
    x, f = orc.make_inputs(450, m, h, i, r)
    fd = [to_dev(a, cuda_device) for a in f]
    xd = to_dev(x, cuda_device)
    yc = ops.contracted_svd_mlp(xd, *fd)
    ys = ops.svd_mlp(xd, *fd)
    torch.cuda.synchronize()
    assert torch.equal(yc, ys)
    assert_close(to_np(yc), orc.svd_mlp(x, *f), what="contracted above 16 tokens")


def test_contracted_reports_range(cuda_device, ops):
    """A row 1000x the typical scale pushes H past fp16 inside the contracted
    unit (H is never stored to global memory): still reported."""
    from svdflash_b200 import _lib
    m, h, r, i = 4, 1024, 300, 2048
    x, f = orc.make_inputs(460, m, h, i, r)
    x = x.copy()
    x[1] *= 1000.0
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    ops.check_device_status(cuda_device)
    ops.contracted_mlp_packed(layer, to_dev(orc.bf16_round(x), cuda_device))
    with pytest.raises(_lib.SvdMlpRangeError):
        ops.check_device_status(cuda_device)
