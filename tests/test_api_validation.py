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
    assert config.MODELS["llama-3.1-8b"]["rank_at_080"] == 2560
    b = config.gate_up_block_params(1024)
    assert isinstance(b, config.GateUpBlocks) and b._asdict()["bn"] == config.GATE_UP_BLOCK_N
    assert b._replace(bn=256).bn == 256
    assert config.fits_smem(config.smem_bytes_gate_up())
    assert config.fits_vmem(config.vmem_bytes_xuv())
    with pytest.raises(ValueError, match="SMEM/TMEM budget exceeds"):
        config.check_budget(config.SMEM_BUDGET_BYTES + 1)
    assert config.tmem_columns_gate_up() <= config.TMEM_COLUMNS


def test_silu_helper_matches_formula():
    x = torch.linspace(-20, 20, 101)
    torch.testing.assert_close(ops.silu(x), x * torch.sigmoid(x))


def test_host_pipeline_argument_checks():
    """HostPipeline refuses a depth that cannot overlap the copies (checked
    before any device buffer or stream is created)."""
    from svdflash_b200.pipeline import HostPipeline
    with pytest.raises(ValueError, match="depth"):
        HostPipeline(lambda x, out: out, (4, 8), (4, 8), device="cuda:0", depth=1)
