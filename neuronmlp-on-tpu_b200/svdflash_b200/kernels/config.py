"""Model table, rank formulas, block descriptors and on-chip budget checks.

Mirrors the ``svdflash_tpu.kernels.config`` API that the reference benches
import (bench/latency.py:23-42, bench/tune.py:135-137,
models/modeling_llama.py:62-73, 367-375).  The TPU's VMEM budget becomes the
B200's per-CTA shared-memory (227 KB) and per-SM TMEM (512 columns) budget of
the tcgen05 kernels; the ``vmem_*`` names are kept as aliases of the
``smem_*`` functions so the reference call sites keep working.
"""
from __future__ import annotations

from typing import NamedTuple

from .ops import low_rank_dim, rank_for_ratio

# Model shapes (hidden_size, intermediate_size, layers, heads, kv heads).
MODELS = {
    "llama-3.1-8b": dict(hidden_size=4096, intermediate_size=14336, num_layers=32, num_heads=32, num_kv_heads=8),
    "llama-3.2-3b": dict(hidden_size=3072, intermediate_size=8192, num_layers=28, num_heads=24, num_kv_heads=8),
    "qwen3-8b": dict(hidden_size=4096, intermediate_size=12288, num_layers=36, num_heads=32, num_kv_heads=8),
    "llama-3-70b": dict(hidden_size=8192, intermediate_size=28672, num_layers=80, num_heads=64, num_kv_heads=8),
}
for _m in MODELS.values():
    _m["rank_at_080"] = low_rank_dim(_m["hidden_size"], _m["intermediate_size"], 0.8)

# Tile shapes of the B200 kernels (rows x K-block x N) and hardware budgets.
BLOCK_M = 128          # tcgen05 MMA M (one TMEM lane per row)
BLOCK_K = 64           # one 128-byte swizzle row of 16-bit elements
GATE_UP_BLOCK_N = 224  # per branch (prefill); two accumulators (gate, up) per tile
DOWN_BLOCK_N = 256
SMEM_BUDGET_BYTES = 232448   # 227 KB opt-in dynamic shared memory per CTA
TMEM_COLUMNS = 512           # 128 lanes x 512 x 32-bit per SM
NUM_SMS_B200 = 148
VMEM_BUDGET_BYTES = SMEM_BUDGET_BYTES

# Down-kernel tile constants kept under the reference names.
XUV_ROW_TILE = BLOCK_M
XUV_INPUT_TILE = BLOCK_K
XUV_RANK_TILE = DOWN_BLOCK_N
XUV_OUTPUT_TILE = DOWN_BLOCK_N


class GateUpBlocks(NamedTuple):
    """Gate/up tiling (bs rows, bh hidden/K block, br rank block, bn ff block)."""
    bs: int
    bh: int
    br: int
    bn: int


def rank_for(model: str, ratio: float) -> int:
    """128-aligned reference rank for a model at a compression ratio."""
    m = MODELS[model]
    return low_rank_dim(m["hidden_size"], m["intermediate_size"], ratio)


def benchmark_rank(model: str, ratio: float) -> int:
    """floor(ratio * in * out / (in + out)): the rank of the benchmark configurations."""
    m = MODELS[model]
    return rank_for_ratio(m["hidden_size"], m["intermediate_size"], ratio)


def gate_up_block_params(rows: int, model: str = "llama-3.1-8b", ratio: float = 0.8) -> GateUpBlocks:
    """The gate/up tiling the B200 kernels use for `rows` tokens."""
    del model, ratio
    return GateUpBlocks(bs=BLOCK_M, bh=BLOCK_K, br=BLOCK_K, bn=GATE_UP_BLOCK_N)


def gate_up_tuning_candidates(rows: int, model: str = "llama-3.1-8b", ratio: float = 0.8, profile=None):
    """Split-K candidates of the gate/up stage (the tunable knob on B200)."""
    del rows, model, ratio, profile
    return [0, 1, 2, 3, 4, 6, 8]


def _stage_smem(bn: int, nb: int, shared_a: bool, stages: int, out_bytes: int) -> int:
    a = BLOCK_M * BLOCK_K * 2
    b = bn * BLOCK_K * 2
    na = 1 if (nb == 1 or shared_a) else 2
    staging = 4 * 2 * 32 * 32 * out_bytes
    bars = (2 * stages + 5) * 8 + 64
    return stages * (na * a + nb * b) + staging + bars + 1024


def _pair_stage_smem(bn: int, nb: int, shared_a: bool, stages: int, out_bytes: int, epi_warps: int) -> int:
    a = BLOCK_M * BLOCK_K * 2
    b = (bn // 2) * BLOCK_K * 2
    na = 1 if (nb == 1 or shared_a) else 2
    staging = epi_warps * 2 * 32 * 32 * out_bytes
    bars = (2 * stages + 5) * 8 + 64
    return stages * (na * a + nb * b) + staging + bars + 1024


def smem_bytes_gate_up(blocks: GateUpBlocks | None = None, r_pad: int = 0, hidden: int = 0) -> int:
    """Shared memory of the gate/up kernels (the larger of its two GEMM stages)."""
    del blocks, r_pad, hidden
    return max(_pair_stage_smem(256, 1, False, 6, 2, 4), _pair_stage_smem(GATE_UP_BLOCK_N, 2, False, 3, 2, 8))


def smem_bytes_xuv(intermediate: int = 0, r_pad: int = 0, hidden: int = 0) -> int:
    del intermediate, r_pad, hidden
    return _stage_smem(256, 1, False, 4, 4)


def smem_bytes_gate_up_down_u(blocks=None, r_g: int = 0, r_d: int = 0, hidden: int = 0) -> int:
    return max(smem_bytes_gate_up(blocks), smem_bytes_xuv())


def tmem_columns_gate_up() -> int:
    return 2 * 256   # two branches of up to 256 columns, one buffer


def fits_smem(nbytes: int) -> bool:
    return nbytes <= SMEM_BUDGET_BYTES


def check_budget(nbytes: int, what: str = "kernel") -> None:
    """Raises the reference's budget error (test_speedup.py:303-317) on overflow."""
    if not fits_smem(nbytes):
        raise ValueError(f"{what}: SMEM/TMEM budget exceeds {SMEM_BUDGET_BYTES} bytes ({nbytes} requested)")


vmem_bytes_gate_up = smem_bytes_gate_up
vmem_bytes_xuv = smem_bytes_xuv
vmem_bytes_gate_up_down_u = smem_bytes_gate_up_down_u
fits_vmem = fits_smem
