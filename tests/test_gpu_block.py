"""The decoder block with its RMSNorm fused (svdmlp_forward_block) against the
CPU oracle's x + svd_mlp(rmsnorm(x)) (bench/e2e_block.py:264-278 without
attention).

The norm weight is folded into u_gate / u_up when the layer is packed and the
row scale rsqrt(mean(x^2) + eps) is applied in the first stage's epilogue, so
the result differs from the unfused chain (a bf16 RMSNorm output fed to the
layer) only by where bf16 rounding happens.

Tolerance.  The inputs' rows span RMS 1e-2 .. 30, so the residual can dwarf
the MLP's contribution and a matrix-wide max-abs/RMS criterion would test
neither.  Each row is checked on its own: |y - ref| <= 2e-2 x RMS(ref - x)
(the north-star criterion applied to the MLP's contribution to that row) plus
the bf16 rounding of the block output (2^-8 |ref|, half an ulp, for the fp32
oracle; a whole ulp, 2^-7 |ref|, between two bf16 outputs); and the relative
Frobenius error of the whole output stays <= 5e-3.  The per-slice sums of
squares the block writes for the next one agree with float64 sums of the bf16
output to 3e-5 relative (fp32 sums of 128 terms).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import svdmlp_oracle as orc
from helpers import to_dev, to_np

pytestmark = pytest.mark.gpu


def _ops():
    from svdflash_b200.kernels import ops
    return ops


def _rows_scaled(seed, m, d):
    """bf16 rows of very different RMS (1e-2 .. 30): the norm has to undo it."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, d), dtype=np.float32)
    x *= np.exp(rng.uniform(np.log(1e-2), np.log(30.0), size=(m, 1))).astype(np.float32)
    return orc.bf16_round(x)


def _norm_weight(seed, d):
    rng = np.random.default_rng(seed)
    return orc.bf16_round(1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32))


def _assert_rows(got, ref, x, what, tol=2e-2, ulp=2.0 ** -8, rel=5e-3):
    g, r, x = (np.asarray(a, dtype=np.float64) for a in (got, ref, x))
    assert np.all(np.isfinite(g)), f"{what}: non-finite outputs"
    rel_fro = np.linalg.norm(g - r) / np.linalg.norm(r)
    assert rel_fro <= rel, f"{what}: rel-Frobenius {rel_fro:.3e} > {rel}"
    contrib = np.sqrt(np.mean((r - x) ** 2, axis=1, keepdims=True))
    excess = np.abs(g - r) - (tol * contrib + ulp * np.abs(r))
    row = int(np.argmax(excess.max(axis=1)))
    assert excess.max() <= 0, (f"{what}: row {row} exceeds its bound by {excess.max():.3e} "
                               f"(row contribution RMS {contrib[row, 0]:.3e})")


def _slice_sumsq(y):
    y = np.asarray(y, dtype=np.float64)
    m, d = y.shape
    parts = -(-d // 128)
    pad = np.zeros((m, parts * 128))
    pad[:, :d] = y
    return (pad * pad).reshape(m, parts, 128).sum(axis=2)


# (M, d, ff, r): the contracted decode schedule (M = 1), the whole-layer decode
# kernel (M <= 16), the weight-streaming kernels (M <= 128) and the tcgen05
# prefill stages; d = 1000 leaves a partial last 128-column slice.
BLOCK_CASES = [
    (1, 1024, 3584, 700),
    (3, 1024, 3584, 700),
    (16, 1000, 2048, 300),
    (40, 1024, 3584, 700),
    (130, 1000, 2048, 300),
    (300, 1024, 3584, 700),
]


@pytest.mark.parametrize("case", BLOCK_CASES)
def test_block_matches_oracle_and_writes_stats(cuda_device, case):
    ops = _ops()
    m, d, ff, r = case
    _, f = orc.make_inputs(300 + m, 1, d, ff, r)
    x = _rows_scaled(310 + m, m, d)
    w = _norm_weight(320 + m, d)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f], norm_weight=to_dev(w, cuda_device))
    xd = to_dev(x, cuda_device)
    xs = ops.row_sumsq(xd)
    np.testing.assert_allclose(to_np(xs), _slice_sumsq(x), rtol=3e-5, atol=1e-30)
    ys = torch.full_like(xs, float("nan"))
    y = ops.svd_block_packed(layer, xd, xs, y_stats=ys, eps=1e-5)
    ops.check_device_status()
    ref = orc.mlp_block(x, w, f, eps=1e-5)
    _assert_rows(to_np(y), ref, x, what=f"block {case}")
    np.testing.assert_allclose(to_np(ys), _slice_sumsq(to_np(y)), rtol=3e-5, atol=1e-30)
    # deterministic: the same call again gives the same bits
    y2 = ops.svd_block_packed(layer, xd, xs, y_stats=torch.empty_like(xs), eps=1e-5)
    torch.testing.assert_close(y2, y, rtol=0, atol=0)


@pytest.mark.parametrize("m", [1, 40, 300])
def test_block_close_to_unfused_chain(cuda_device, m):
    """Fused block vs rmsnorm kernel + layer with the residual in its epilogue."""
    ops = _ops()
    d, ff, r = 1024, 3584, 700
    _, f = orc.make_inputs(400 + m, 1, d, ff, r)
    x = _rows_scaled(410 + m, m, d)
    w = _norm_weight(420 + m, d)
    fd = [to_dev(a, cuda_device) for a in f]
    xd, wd = to_dev(x, cuda_device), to_dev(w, cuda_device)
    fused = ops.svd_block_packed(ops.pack_svd_layer(*fd, norm_weight=wd), xd, ops.row_sumsq(xd))
    plain = ops.svd_mlp_packed(ops.pack_svd_layer(*fd), ops.rmsnorm(xd, wd, 1e-5), residual=xd)
    _assert_rows(to_np(fused), to_np(plain), x, what=f"fused vs unfused m={m}", ulp=2.0 ** -7)


def test_fused_stack_eager_graph_and_mixed(cuda_device):
    from svdflash_b200.models import MlpBlockStack, SvdLlamaMLP, SvdMlpBlock
    d, ff, r, layers = 1024, 2048, 300, 4
    facs = [orc.make_inputs(500 + l, 1, d, ff, r)[1] for l in range(layers)]
    norms = [_norm_weight(510 + l, d) for l in range(layers)]
    dev = lambda a: to_dev(a, cuda_device)  # noqa: E731
    fused = MlpBlockStack([SvdMlpBlock(*[dev(a) for a in f], dev(w)) for f, w in zip(facs, norms)])
    # blocks 0 and 1 fused, 2 unfused, 3 fused again (its statistics recomputed)
    mixed = MlpBlockStack(
        [SvdMlpBlock(*[dev(a) for a in facs[0]], dev(norms[0])),
         SvdMlpBlock(*[dev(a) for a in facs[1]], dev(norms[1])),
         SvdLlamaMLP(*[dev(a) for a in facs[2]]),
         SvdMlpBlock(*[dev(a) for a in facs[3]], dev(norms[3]))],
        [None, None, dev(norms[2]), None])
    for m in (1, 5, 200):
        x = _rows_scaled(520 + m, m, d)
        # the residual stream is bf16 between blocks, in the oracle chain too;
        # where the GPU's and the oracle's block output straddle a bf16
        # rounding boundary they differ by an ulp, which the later blocks
        # carry along: up to one ulp per block on top of the MLP criterion
        ref = x
        for f, w in zip(facs, norms):
            ref = orc.bf16_round(orc.mlp_block(ref, w, f, eps=1e-5))
        y = fused(dev(x))
        bound = dict(tol=4e-2, rel=1e-2, ulp=layers * 2.0 ** -7)
        _assert_rows(to_np(y), ref, x, what=f"fused stack m={m}", **bound)
        _assert_rows(to_np(mixed(dev(x))), ref, x, what=f"mixed stack m={m}", **bound)
        fused.capture(m, d, cuda_device)
        yg = fused.replay(dev(x))
        torch.cuda.synchronize()
        torch.testing.assert_close(yg, y, rtol=0, atol=0)
    _ops().check_device_status()


def test_block_argument_errors(cuda_device):
    ops = _ops()
    d, ff, r = 256, 512, 64
    _, f = orc.make_inputs(600, 1, d, ff, r)
    fd = [to_dev(a, cuda_device) for a in f]
    plain = ops.pack_svd_layer(*fd)
    x = to_dev(_rows_scaled(601, 4, d), cuda_device)
    xs = ops.row_sumsq(x)
    with pytest.raises(ValueError):
        ops.svd_block_packed(plain, x, xs)           # packed without its norm weight
    normed = ops.pack_svd_layer(*fd, norm_weight=torch.ones(d, device=cuda_device, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        ops.svd_block_packed(normed, x, xs, out=x)   # y must not alias x
    with pytest.raises(ValueError):
        ops.pack_svd_layer(*fd, norm_weight=torch.ones(d + 1, device=cuda_device))
    with pytest.raises(ValueError):
        ops.svd_block_packed(normed, x, xs[:, :1].contiguous())  # too few slices per row


@pytest.mark.parametrize("m", [3, 16])
def test_block_on_forced_whole_layer_kernel(cuda_device, m):
    """The plain whole-layer decode schedule (default only at one token, where
    it is contracted) with the fused norm: forced for 3 and 16 tokens."""
    from svdflash_b200 import _lib
    ops = _ops()
    lib = _lib.load()
    d, ff, r = 1024, 3584, 700
    _, f = orc.make_inputs(700 + m, 1, d, ff, r)
    x = _rows_scaled(710 + m, m, d)
    w = _norm_weight(720 + m, d)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f], norm_weight=to_dev(w, cuda_device))
    xd = to_dev(x, cuda_device)
    xs = ops.row_sumsq(xd)
    ys = torch.full_like(xs, float("nan"))
    try:
        assert lib.svdmlp_set_layer_decode(16) == 0
        y = ops.svd_block_packed(layer, xd, xs, y_stats=ys)
        torch.cuda.synchronize()
    finally:
        lib.svdmlp_set_layer_decode(-1)
    ops.check_device_status()
    _assert_rows(to_np(y), orc.mlp_block(x, w, f, eps=1e-5), x, what=f"forced whole-layer block m={m}")
    np.testing.assert_allclose(to_np(ys), _slice_sumsq(to_np(y)), rtol=3e-5, atol=1e-30)


@pytest.mark.parametrize("m", [1, 4, 1024])
def test_block_at_the_8b_shape(cuda_device, m):
    """Config 3's block (Llama-3-8B, ratio 0.9, r = 2867) with the norm fused:
    one token (contracted whole-layer kernel), four tokens (plain whole-layer
    kernel) and 1024 tokens (CTA-pair GEMMs), full output, per-row criterion,
    with the statistics the block writes for the next one."""
    import math
    ops = _ops()
    d, ff, r = 4096, 14336, 2867
    g = torch.Generator(device=cuda_device)
    g.manual_seed(800 + m)

    def mat(rows, cols):
        return (torch.randn(rows, cols, generator=g, device=cuda_device) / math.sqrt(rows)).to(torch.bfloat16)

    fd = [mat(d, r), mat(r, ff), mat(d, r), mat(r, ff), mat(ff, r), mat(r, d)]
    f = [to_np(t) for t in fd]
    w = _norm_weight(810 + m, d)
    x = _rows_scaled(820 + m, m, d)
    layer = ops.pack_svd_layer(*fd, norm_weight=to_dev(w, cuda_device))
    del fd
    xd = to_dev(x, cuda_device)
    xs = ops.row_sumsq(xd)
    ys = torch.full_like(xs, float("nan"))
    y = ops.svd_block_packed(layer, xd, xs, y_stats=ys)
    ops.check_device_status()
    _assert_rows(to_np(y), orc.mlp_block(x, w, f, eps=1e-5), x, what=f"8B block m={m}")
    np.testing.assert_allclose(to_np(ys), _slice_sumsq(to_np(y)), rtol=3e-5, atol=1e-30)
