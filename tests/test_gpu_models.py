"""GPU tests of the model hook, the launcher-name API, the block stack (eager
and CUDA graph) and the single-GPU tensor-parallel path, against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import svdmlp_oracle as orc
from helpers import assert_close, to_dev, to_np

pytestmark = pytest.mark.gpu


def test_svd_module_3d_input_and_linear_order(cuda_device):
    from svdflash_b200.models import SvdLlamaMLP
    b, s, h, r, i = 2, 70, 256, 96, 512
    x, f = orc.make_inputs(31, b * s, h, i, r)
    fd = [to_dev(a, cuda_device) for a in f]
    mod = SvdLlamaMLP(*fd)
    y = mod(to_dev(x, cuda_device).reshape(b, s, h))
    assert tuple(y.shape) == (b, s, h)
    ref = orc.svd_mlp(x, *f)
    assert_close(to_np(y).reshape(b * s, h), ref, what="module")
    # torch.nn.Linear order: *_v_proj [r, in] (first factor^T), *_u_proj [out, r]
    mod2 = SvdLlamaMLP.from_torch_linear_factors(fd[0].t(), fd[1].t(), fd[2].t(), fd[3].t(), fd[4].t(), fd[5].t())
    y2 = mod2(to_dev(x, cuda_device))
    torch.testing.assert_close(y2, y.reshape(b * s, h), rtol=0, atol=0)


def test_launcher_names(cuda_device):
    from svdflash_b200.kernels import launchers
    s, h, r, i = 40, 128, 64, 256
    x, f = orc.make_inputs(32, s, h, i, r)
    ug, vg, uu, vu, ud, vd = [to_dev(a, cuda_device) for a in f]
    xd = to_dev(x, cuda_device)
    y = launchers.svd_mlp_with_fused_kernel(xd, uu, vu, ug, vg, ud, vd)   # up-before-gate order
    assert_close(to_np(y), orc.svd_mlp(x, *f), what="svd_mlp_with_fused_kernel")
    ht = launchers.fused_mlp_up_T(xd, ug, vg, uu, vu)
    assert tuple(ht.shape) == (i, s)
    assert ht.t().is_contiguous()  # a view of the row-major [S, I] output, no copy
    y2 = launchers.fused_three_mm_XTUV(ht, ud, vd)
    hb = orc.bf16_round(orc.fused_gate_up(x, *f[:4]))
    assert_close(to_np(y2), orc.fused_xuv(hb, f[4], f[5]), what="XTUV")
    # a row-major [I, S] activation (any other producer) gives the same result
    y2c = launchers.fused_three_mm_XTUV(ht.contiguous(), ud, vd)
    assert torch.equal(y2c, y2)
    y3 = launchers.nki_mm(xd, uu.t(), vu.t(), ug.t(), vg.t(), ud.t(), vd.t())
    assert_close(to_np(y3), orc.svd_mlp(x, *f), what="nki_mm")
    wg, wu, wd = orc.make_dense(33, h, i)
    yd = launchers.nki_baseline(xd, to_dev(wu, cuda_device).t(), to_dev(wg, cuda_device).t(), to_dev(wd, cuda_device).t())
    assert_close(to_np(yd), orc.dense_mlp(x, wg, wu, wd), what="nki_baseline")


def test_block_stack_eager_and_graph(cuda_device):
    from svdflash_b200.models import MlpBlockStack, SvdLlamaMLP
    m, h, r, i, layers = 200, 256, 72, 512, 3
    rng = np.random.default_rng(40)
    x = orc.bf16_round(rng.standard_normal((m, h), dtype=np.float32))
    facs, norms = [], []
    for l in range(layers):
        _, f = orc.make_inputs(41 + l, 1, h, i, r)
        facs.append(f)
        norms.append(orc.bf16_round(1 + 0.02 * rng.standard_normal(h, dtype=np.float32)))
    stack = MlpBlockStack([SvdLlamaMLP(*[to_dev(a, cuda_device) for a in f]) for f in facs],
                          [to_dev(w, cuda_device) for w in norms], eps=1e-5)
    ref = x
    for f, w in zip(facs, norms):
        ref = orc.mlp_block(ref, w, f, eps=1e-5)
    y = stack(to_dev(x, cuda_device))
    assert_close(to_np(y), ref, rel=1e-2, max_abs_rms=4e-2, what="stack eager (bf16 residual stream)")
    stack.capture(m, h, cuda_device)
    yg = stack.replay(to_dev(x, cuda_device))
    torch.cuda.synchronize()
    torch.testing.assert_close(yg, y, rtol=0, atol=0)


def test_tensor_parallel_single_rank(cuda_device):
    from svdflash_b200.tp import TensorParallelSvdMlp
    m, h, r, i = 150, 256, 100, 512
    x, f = orc.make_inputs(50, m, h, i, r)
    tp = TensorParallelSvdMlp(*[to_dev(a, cuda_device) for a in f], rank=0, world=1)
    y = tp(to_dev(x, cuda_device))
    assert_close(to_np(y), orc.svd_mlp(x, *f), what="tp world=1")


@pytest.mark.parametrize("world,dtype", [(2, "float32"), (2, "float16"), (8, "float16")])
def test_tensor_parallel_shards_summed_on_one_gpu(cuda_device, world, dtype):
    """`world` ff-shards run on one GPU; their partials (fp32, or fp16 summed
    one rank after another in fp16, as a ring all-reduce of ncclHalf rounds)
    reproduce the full layer through down_finish; each shard's partial
    matches the oracle's shard arithmetic."""
    from svdflash_b200.kernels import ops
    from svdflash_b200.tp import TensorParallelSvdMlp
    m, h, r, i = 128, 1024, 700, 3584
    x, f = orc.make_inputs(51, m, h, i, r)
    fd = [to_dev(a, cuda_device) for a in f]
    xd = to_dev(x, cuda_device)
    td = getattr(torch, dtype)
    parts = []
    shards = [TensorParallelSvdMlp(*fd, rank=p, world=world, reduce_dtype=td) for p in range(world)]
    for sh in shards:
        buf = sh._partial_buffer(m, cuda_device).clone()
        ops.forward_partial_packed(sh.layer, xd, buf[:, :sh.r_d])
        assert buf.dtype == td
        parts.append(buf)
    total = parts[0].clone()
    for p in parts[1:]:
        total = total + p  # rounds to the partial's dtype after every rank
    y = ops.down_finish_packed(shards[0].layer, total[:, :r])
    assert_close(to_np(y), orc.svd_mlp(x, *f), what=f"tp {world} shards ({dtype}) on one gpu")
    for p, sh in enumerate(shards[:2]):
        want = orc.shard_partial(x, orc.shard_factors(f, p, world))
        got = to_np(parts[p][:, :r])
        assert orc.error_metrics(got, want)["rel_fro"] < 5e-3


@pytest.mark.parametrize("world", [2, 8])
def test_tensor_parallel_split_mode_on_one_gpu(cuda_device, world):
    """The all-gather split of the replicated stages, `world` ranks emulated on
    one GPU: X.[u_g|u_u] per row block (all-gathered), stages 2-3 per ff shard
    on all rows, the fp16 partials summed rank after rank (reduce-scatter by
    rows), .v_down (+ residual) per row block (all-gathered): the full layer."""
    from svdflash_b200.kernels import ops
    from svdflash_b200.tp import TensorParallelSvdMlp
    m, h, r, i = 128, 1024, 700, 3584
    x, f = orc.make_inputs(52, m, h, i, r)
    res = orc.bf16_round(np.random.default_rng(53).standard_normal((m, h), dtype=np.float32))
    fd = [to_dev(a, cuda_device) for a in f]
    xd, rd = to_dev(x, cuda_device), to_dev(res, cuda_device)
    shards = [TensorParallelSvdMlp(*fd, rank=p, world=world, mode="split") for p in range(world)]
    rows = m // world
    xu = torch.cat([ops.xu_project_packed(shards[p].layer, xd[p * rows:(p + 1) * rows]) for p in range(world)])
    xu_full = ops.xu_project_packed(shards[0].layer, xd)
    torch.cuda.synchronize()
    assert torch.equal(xu, xu_full) or orc.error_metrics(to_np(xu), to_np(xu_full))["rel_fro"] < 1e-3
    total = None
    for sh in shards:
        buf = sh._partial_buffer(m, cuda_device).clone()  # 16-byte rows (r padded to 8)
        ops.partial_from_xu_packed(sh.layer, xu, buf[:, :r])
        total = buf if total is None else total + buf
    ys = [ops.down_finish_packed(shards[p].layer, total[p * rows:(p + 1) * rows, :r],
                                 residual=rd[p * rows:(p + 1) * rows]) for p in range(world)]
    y = torch.cat(ys)
    assert_close(to_np(y), res + orc.svd_mlp(x, *f), what=f"tp split mode, {world} ranks on one gpu")
    ops.check_device_status(cuda_device)


def test_decode_sizes_split_k(cuda_device):
    """M <= 128 runs the one-CTA split-K kernels (config 2 regime, small dims)."""
    from svdflash_b200.kernels import ops
    h, r, i = 1024, 764, 3584
    _, f = orc.make_inputs(60, 1, h, i, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    for m in (1, 8, 32, 128):
        x = orc.bf16_round(np.random.default_rng(m).standard_normal((m, h), dtype=np.float32))
        y = ops.svd_mlp_packed(layer, to_dev(x, cuda_device))
        assert_close(to_np(y), orc.svd_mlp(x, *f), what=f"decode m={m}")
    ops.check_device_status(cuda_device)


@pytest.mark.parametrize("m", [17, 40, 100, 128])
def test_per_stage_decode_forced_splits(cuda_device, m):
    """Per-stage decode kernels (16 < M <= 128) with split-K forced on every
    stage, the dual gate/up included: above 16 tokens all splits of a tile sum
    a share of its token rows; outputs go through the staged row stores, with
    a partial last 16-token chunk (m = 40, 100), a rank that leaves a scalar
    tail at N (763), and the residual epilogue.  Matches the oracle, repeats
    bitwise, and agrees with the unsplit run."""
    from svdflash_b200 import _lib
    from svdflash_b200.kernels import ops
    lib = _lib.load()
    h, r, i = 1024, 763, 3584
    x, f = orc.make_inputs(140 + m, m, h, i, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    xd = to_dev(x, cuda_device)
    res = orc.bf16_round(np.random.default_rng(m).standard_normal((m, h), dtype=np.float32))
    rd = to_dev(res, cuda_device)
    ref = orc.svd_mlp(x, *f)
    try:
        y0 = ops.svd_mlp_packed(layer, xd, residual=rd)
        for splits in (2, 3, 5):
            for st in range(4):
                assert lib.svdmlp_set_split_override(st, splits) == 0
            y1 = ops.svd_mlp_packed(layer, xd, residual=rd)
            y2 = ops.svd_mlp_packed(layer, xd, residual=rd)
            torch.cuda.synchronize()
            assert torch.equal(y1, y2), f"m={m} splits={splits}: runs differ"
            assert_close(to_np(y1), res + ref, what=f"per-stage decode m={m} splits={splits}")
            from helpers import assert_close_bf16_output
            assert_close_bf16_output(to_np(y1), to_np(y0), what=f"split {splits} vs planner m={m}")
    finally:
        for st in range(4):
            lib.svdmlp_set_split_override(st, 0)
    ops.check_device_status(cuda_device)


@pytest.mark.parametrize("m", [1, 5, 16, 17, 64])
def test_whole_layer_decode_kernel(cuda_device, m):
    """The one-launch whole-layer decode kernel (forced up to M = 64, both token
    tile widths) matches the oracle and the four per-stage kernels, with and
    without a residual, and gives the same bits with the overlapped
    (programmatic dependent) launch turned off."""
    from svdflash_b200 import _lib
    from svdflash_b200.kernels import ops
    lib = _lib.load()
    h, r, i = 4096, 2867, 14336
    x, f = orc.make_inputs(90 + m, m, h, i, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    xd = to_dev(x, cuda_device)
    res = orc.bf16_round(np.random.default_rng(m).standard_normal((m, h), dtype=np.float32))
    rd = to_dev(res, cuda_device)
    try:
        assert lib.svdmlp_set_layer_decode(64) == 0
        y1 = ops.svd_mlp_packed(layer, xd)
        y1r = ops.svd_mlp_packed(layer, xd, residual=rd)
        y1b = ops.svd_mlp_packed(layer, xd)
        assert lib.svdmlp_set_decode_overlap(0) == 0
        y1s = ops.svd_mlp_packed(layer, xd)
        lib.svdmlp_set_decode_overlap(1)
        lib.svdmlp_set_layer_decode(0)
        y0 = ops.svd_mlp_packed(layer, xd)
    finally:
        lib.svdmlp_set_layer_decode(-1)
        lib.svdmlp_set_decode_overlap(1)
    torch.cuda.synchronize()
    ops.check_device_status(cuda_device)
    ref = orc.svd_mlp(x, *f)
    assert_close(to_np(y1), ref, what=f"layer decode m={m}")
    assert_close(to_np(y1r), res + ref, what=f"layer decode + residual m={m}")
    assert torch.equal(y1, y1b), "repeated launches differ"
    # a plain launch (no programmatic dependent launch): identical bits
    assert torch.equal(y1, y1s), "the overlapped launch changes the result"
    from helpers import assert_close_bf16_output
    assert_close_bf16_output(to_np(y1), to_np(y0), what=f"layer decode vs per-stage m={m}")


@pytest.mark.parametrize("m", [129, 300, 700])
def test_prefill_chain_matches_unchained(cuda_device, m):
    """Prefill layers run their four GEMMs as a chain (per-M-tile counters in
    place of whole-launch waits, M-tile groups in the unit order).  Chained
    stages are unsplit; with split-K turned off on the unchained side too the
    tiles and their accumulation order are the same, so the outputs are
    bit-identical; repeated calls re-arm the counters; partial and odd M-tile
    counts and the residual epilogue are covered."""
    from svdflash_b200 import _lib
    from svdflash_b200.kernels import ops
    lib = _lib.load()
    h, r, i = 1024, 700, 3584
    x, f = orc.make_inputs(120 + m, m, h, i, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    xd = to_dev(x, cuda_device)
    res = orc.bf16_round(np.random.default_rng(m).standard_normal((m, h), dtype=np.float32))
    rd = to_dev(res, cuda_device)
    try:
        for st in range(4):
            assert lib.svdmlp_set_split_override(st, 1) == 0
        assert lib.svdmlp_set_prefill_chain(2) == 0
        ys = [ops.svd_mlp_packed(layer, xd) for _ in range(3)]
        yr = ops.svd_mlp_packed(layer, xd, residual=rd)
        assert lib.svdmlp_set_prefill_chain(3) == 0
        y1 = ops.svd_mlp_packed(layer, xd)
        assert lib.svdmlp_set_prefill_chain(0) == 0
        y0 = ops.svd_mlp_packed(layer, xd)
        y0r = ops.svd_mlp_packed(layer, xd, residual=rd)
    finally:
        lib.svdmlp_set_prefill_chain(0)
        for st in range(4):
            lib.svdmlp_set_split_override(st, 0)
    torch.cuda.synchronize()
    ops.check_device_status(cuda_device)
    for k, y in enumerate(ys):
        assert torch.equal(y, y0), f"chained call {k} differs from the unchained path"
    assert torch.equal(y1, y0), "three M-tile groups differ from the unchained path"
    assert torch.equal(yr, y0r), "chained residual epilogue differs"
    assert_close(to_np(ys[0]), orc.svd_mlp(x, *f), what=f"chained prefill m={m}")


def test_host_pipeline_matches_direct_calls(cuda_device):
    """HostPipeline (uploads, layer calls and downloads on three streams with
    double-buffered device tensors) returns exactly the direct calls' outputs
    for a sequence of distinct host batches, including one longer than the
    buffer depth and a second run on the same pipeline."""
    from svdflash_b200.kernels import ops
    from svdflash_b200.pipeline import HostPipeline
    m, h, r, i = 300, 1024, 700, 3584
    _, f = orc.make_inputs(170, m, h, i, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    rng = np.random.default_rng(171)
    xs = [torch.from_numpy(orc.bf16_round(rng.standard_normal((m, h), dtype=np.float32))).to(torch.bfloat16)
          for _ in range(5)]
    ref = [ops.svd_mlp_packed(layer, x.to(cuda_device)).cpu() for x in xs]
    pipe = HostPipeline(lambda x, out: ops.svd_mlp_packed(layer, x, out=out), (m, h), (m, h), device=cuda_device)
    for _ in range(2):
        x_host = [x.pin_memory() for x in xs]
        y_host = [torch.empty(m, h, dtype=torch.bfloat16).pin_memory() for _ in xs]
        pipe.run(x_host, y_host)
        torch.cuda.current_stream(cuda_device).synchronize()
        for k, (y, yr) in enumerate(zip(y_host, ref)):
            assert torch.equal(y, yr), f"batch {k} differs from the direct call"
    with pytest.raises(ValueError):
        HostPipeline(lambda x, out: x, (m, h), (m, h), device=cuda_device, depth=1)


@pytest.mark.parametrize("m", [40, 128])
def test_pair_gemms_below_default_threshold(cuda_device, m):
    """With the pair threshold lowered (svdmlp_set_pair_min_m), decode-sized
    layers run on the CTA-pair GEMMs (one partial 256-row M-tile) and still
    match the oracle and the decode kernels' result; the workspace sized for
    the default threshold already covers their split-K partials."""
    from svdflash_b200 import _lib
    from svdflash_b200.kernels import ops
    from helpers import assert_close_bf16_output
    lib = _lib.load()
    h, r, i = 1024, 700, 3584
    x, f = orc.make_inputs(180 + m, m, h, i, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    xd = to_dev(x, cuda_device)
    y0 = ops.svd_mlp_packed(layer, xd)
    try:
        assert lib.svdmlp_set_pair_min_m(17) == 0
        y1 = ops.svd_mlp_packed(layer, xd)
    finally:
        lib.svdmlp_set_pair_min_m(-1)
    torch.cuda.synchronize()
    ops.check_device_status(cuda_device)
    assert_close(to_np(y1), orc.svd_mlp(x, *f), what=f"pair GEMMs m={m}")
    assert_close_bf16_output(to_np(y1), to_np(y0), what=f"pair GEMMs vs decode kernels m={m}")
