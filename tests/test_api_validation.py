"""Host-side validation of the operator API, with the reference's error
types and messages (test_speedup.py:37-49; snapshot test cases
tests_test_speedup_migration.py.before:122-132)."""
from __future__ import annotations

import pytest
import torch

from svdflash_b200.kernels import config, ops


def t(*shape, dtype=torch.bfloat16):
    return torch.zeros(*shape, dtype=dtype)


def test_non_2d_and_empty_inputs():
    with pytest.raises(ValueError, match="nonempty 2D"):
        ops.svd_mlp(t(4), t(4, 3), t(3, 5), t(4, 3), t(3, 5), t(5, 3), t(3, 4))
    with pytest.raises(ValueError, match="nonempty 2D"):
        ops.fused_gate_up(t(0, 4), t(4, 3), t(3, 5), t(4, 3), t(3, 5))


def test_mixed_and_unsupported_dtypes():
    with pytest.raises(TypeError, match="same dtype"):
        ops.xuv_matmul(t(2, 4), t(4, 3, dtype=torch.float32), t(3, 4))
    with pytest.raises(TypeError, match="supported dtypes"):
        ops.xuv_matmul(t(2, 4, dtype=torch.float16), t(4, 3, dtype=torch.float16), t(3, 4, dtype=torch.float16))


def test_cpu_tensors_are_rejected_loudly():
    with pytest.raises(ValueError, match="CUDA"):
        ops.xuv_matmul(t(2, 4), t(4, 3), t(3, 4))


def test_modes_without_cpu_path():
    with pytest.raises(NotImplementedError):
        ops._check_modes(True, True, torch.bfloat16)
    with pytest.raises(NotImplementedError):
        ops._check_modes(False, False, torch.float32)
    ops._check_modes(True, False, torch.float32)


def test_positive_integer_messages():
    with pytest.raises(ValueError, match="positive integer"):
        ops._positive("bs", 0)
    with pytest.raises(ValueError, match="positive integer"):
        ops._positive("bs", True)


def test_rank_formulas():
    assert ops.low_rank_dim(4096, 14336, 0.8) == 2560
    assert ops.low_rank_dim(3072, 8192, 0.8) == 1792
    assert ops.rank_for_ratio(4096, 14336, 0.9) == 2867
    assert config.rank_for("llama-3.1-8b", 0.9) == 2816
    assert config.benchmark_rank("llama-3-70b", 0.8) == 5097


def test_config_tables_and_budget():
    m8 = config.MODELS["llama-3.1-8b"]
    assert isinstance(m8, config.ModelShape) and m8.hidden_size == 4096 and m8.rank_at_080 == 2560
    assert config.rank_for(m8, 0.9) == config.rank_for("llama-3.1-8b", 0.9) == 2816
    b = config.gate_up_block_params(1024, m8, 0.9)
    # the compiled prefill tile: 256-row CTA pairs, 256 ff columns per branch,
    # 64-wide K blocks; the split count is the library planner's
    assert isinstance(b, config.GateUpBlocks) and (b.bs, b.bh, b.br, b.bn) == (256, 64, 64, 256)
    assert b.splits == config.stage_plan(config.STAGE_GATE_UP, 1024, 14336, 2816).splits
    assert b._replace(bn=256).bn == 256 and set(b._asdict()) == {"bs", "bh", "br", "bn", "splits"}
    d = config.gate_up_block_params(1, m8, 0.9)   # decode: 16-token tiles over 128-row weight panels
    assert (d.bs, d.bn) == (16, 128)
    assert config.gate_up_block_params(100, m8, 0.9).bs == 128
    t = config.tile_info(config.STAGE_GATE_UP, 1024)
    assert config.smem_bytes_gate_up() == t.smem_bytes
    # the layout formula reproduces the compiled kernel's shared memory
    assert config._pair_smem(t.tile_cols, 2, False, t.stages, 2, 8, 2) == t.smem_bytes
    assert config.fits_smem(config.smem_bytes_gate_up())
    assert config.fits_vmem(config.vmem_bytes_xuv())
    with pytest.raises(ValueError, match="SMEM/TMEM budget exceeds"):
        config.check_budget(config.SMEM_BUDGET_BYTES + 1)
    assert config.tmem_columns_gate_up() <= config.TMEM_COLUMNS
    # a tile the SM cannot hold is refused with the reference's budget error
    with pytest.raises(ValueError, match="SMEM/TMEM budget exceeds"):
        config.check_gate_up_blocks(b._replace(bn=512))
    with pytest.raises(ValueError, match="positive integer"):
        config.check_gate_up_blocks(b._replace(bs=0))
    config.check_gate_up_blocks(b)


def test_tuning_candidates_are_real_split_counts():
    m8 = config.MODELS["llama-3.1-8b"]
    cands = config.gate_up_tuning_candidates(1024, m8, 0.9)
    base = config.gate_up_block_params(1024, m8, 0.9)
    assert cands[0].splits == max(1, base.splits)
    k_blocks = -(-2816 // 64)
    assert all(-(-k_blocks // c.splits) >= 8 for c in cands)   # at least 8 k-blocks per CTA-pair split
    assert len({c.splits for c in cands}) == len(cands) >= 2
    assert all((c.bs, c.bn) == (base.bs, base.bn) for c in cands)
    quick = config.gate_up_tuning_candidates(1024, m8, 0.9, profile="quick")
    assert 1 <= len(quick) <= 3


def test_reference_package_facade_exports():
    """The import lines of the reference's benches and model resolve to the
    B200 operators (bench/latency.py:23-42, bench/e2e_block.py:40-48,
    bench/all_mlp_layers.py:21-31, bench/tune.py:20-27)."""
    from svdflash_tpu.kernels import config as c
    from svdflash_tpu.kernels.config import (  # noqa: F401
        MODELS, XUV_INPUT_TILE, XUV_OUTPUT_TILE, XUV_RANK_TILE, XUV_ROW_TILE, GateUpBlocks, ModelShape, fits_vmem,
        gate_up_block_params, gate_up_tuning_candidates, rank_for, vmem_bytes_gate_up, vmem_bytes_gate_up_down_u,
        vmem_bytes_xuv)
    from svdflash_tpu.kernels.pallas_ops import (contracted_svd_mlp, dense_matmul, dense_mlp, fused_gate_up,
                                                 svd_mlp, xuv_matmul)
    from svdflash_tpu.kernels.reference import (dense_mlp_ref, fused_gate_up_ref, fused_xuv_ref, low_rank_dim,
                                                silu, svd_mlp_ref)  # noqa: F401
    from svdflash_tpu.models.hf_svd import checkpoint_metadata, load_mlp_factors, validate_factor_shapes  # noqa: F401
    from svdflash_tpu.test_speedup import (_positive, get_fused_mlp_up_T_params,  # noqa: F401
                                           get_fused_three_mm_XTUV_params, nki_matmul_fully_optimized_,
                                           svd_mlp_with_fused_kernel)
    assert svd_mlp is ops.svd_mlp and contracted_svd_mlp is ops.contracted_svd_mlp and c.MODELS is config.MODELS
    assert fused_gate_up is ops.fused_gate_up and xuv_matmul is ops.xuv_matmul and dense_mlp is ops.dense_mlp
    assert dense_matmul is ops.dense_matmul and low_rank_dim(4096, 14336, 0.8) == 2560
    p = get_fused_mlp_up_T_params(1024)
    assert (p["tile_rows"], p["tile_cols"]) == (256, 256)
    with pytest.raises(ValueError, match="positive integer"):
        get_fused_three_mm_XTUV_params(0)


def test_silu_helper_matches_formula():
    x = torch.linspace(-20, 20, 101)
    torch.testing.assert_close(ops.silu(x), x * torch.sigmoid(x))


def test_host_pipeline_argument_checks():
    """HostPipeline refuses a depth that cannot overlap the copies (checked
    before any device buffer or stream is created)."""
    from svdflash_b200.pipeline import HostPipeline
    with pytest.raises(ValueError, match="depth"):
        HostPipeline(lambda x, out: out, (4, 8), (4, 8), device="cuda:0", depth=1)


def test_peer_buffer_layout_and_arguments():
    """Peer-memory layout arithmetic and the argument checks that run before
    any CUDA call (the collectives themselves are GPU tests)."""
    from svdflash_b200.peer import PeerBuffer, layout
    offs, total = layout([100, 0, 4096, 1], 32 * 1024)
    assert offs[0] == 32 * 1024 and all(o % 256 == 0 for o in offs)
    assert offs[1] >= offs[0] + 100 and offs[2] >= offs[1] and offs[3] >= offs[2] + 4096
    assert total % 256 == 0 and total >= offs[3] + 1
    with pytest.raises(ValueError):
        PeerBuffer(1 << 20, rank=0, world=9)
    with pytest.raises(ValueError):
        PeerBuffer(1 << 20, rank=2, world=2)


def test_fused_exchange_slot_checks():
    """The fused exchange's slot geometry and the checks PeerBuffer makes
    before any CUDA call, on a buffer object that maps nothing."""
    import torch
    from svdflash_b200 import _build, _lib
    from svdflash_b200.peer import PeerBuffer, layout
    if _build.is_stale():
        _build.build()
    pb = PeerBuffer.__new__(PeerBuffer)  # the arithmetic only: no allocation, no peers
    pb.lib, pb.world, pb.rank = _lib.load(), 2, 0
    pb.signal_bytes = int(pb.lib.svdmlp_peer_signal_bytes())
    pb.device = torch.device("cuda", 0)
    slot_rows, ld = 256, 2872
    n = pb.slots_bytes(slot_rows, ld)
    assert n == 2 * 2 * slot_rows * ld * 2          # two sets of one [slot_rows, ld] fp16 slot per rank
    (off,), pb.nbytes = layout([n], pb.signal_bytes)
    pb.check_slots(off, slot_rows, 1, ld)            # any m up to slot_rows
    pb.check_slots(off, slot_rows, slot_rows, ld)
    for bad in ((off, slot_rows, slot_rows + 1, ld),  # more rows than a slot holds
                (off, slot_rows, 0, ld),
                (off + 8, slot_rows, 4, ld),          # misaligned
                (0, slot_rows, 4, ld),                # in the signal area
                (off, slot_rows + 1, 4, ld),          # slots past the buffer
                (off, slot_rows, 4, ld + 4)):         # row stride not a multiple of 8
        with pytest.raises(ValueError):
            pb.check_slots(*bad)
    out = torch.empty((4, ld), dtype=torch.float32)
    with pytest.raises(ValueError):                  # fp32 out: refused before the call
        pb.sum_f16(off, slot_rows, 4, ld, ld, out)
    with pytest.raises(ValueError):                  # c not a multiple of 8
        pb.sum_f16(off, slot_rows, 4, 2867, ld, torch.empty((4, ld), dtype=torch.float16))
