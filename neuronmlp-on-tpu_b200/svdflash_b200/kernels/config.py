"""Model table, rank formulas, tile plans and on-chip budget checks.

Mirrors the ``svdflash_tpu.kernels.config`` API that the reference benches
and model import (bench/latency.py:23-42, bench/tune.py:20-26,
bench/all_mlp_layers.py:21-31, models/modeling_llama.py:62-73, 355-375):
``MODELS`` maps names to ``ModelShape`` records, ``rank_for(model, ratio)``
and ``gate_up_block_params(rows, model, ratio)`` take such a record, and
``GateUpBlocks`` is the NamedTuple the benches ``_replace`` and ``_asdict``.

On B200 the TPU's VMEM budget becomes the per-CTA shared-memory (227 KB) and
per-SM tensor-memory (512 columns) budget of the tcgen05 kernels.  The
numbers here are not a model of the hardware: tile shapes, pipeline depths,
shared-memory bytes and split-K plans come from the compiled kernels and the
library's own planner (``svdmlp_tile_info``, ``svdmlp_plan_info``), so what a
bench or tuner reads is what runs.  The ``vmem_*`` names are kept as aliases
of the ``smem_*`` functions for the reference's call sites.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple, Optional, Union

from .. import _lib
from .ops import low_rank_dim, rank_for_ratio


class ModelShape(NamedTuple):
    """Shape of a model's MLP (the reference's ``kernels.config`` record)."""
    name: str
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    rank_at_080: int


def _shape(name, hidden, inter, layers, heads, kv_heads) -> ModelShape:
    return ModelShape(name, hidden, inter, layers, heads, kv_heads, low_rank_dim(hidden, inter, 0.8))


MODELS = {
    "llama-3.1-8b": _shape("llama-3.1-8b", 4096, 14336, 32, 32, 8),
    "llama-3.2-3b": _shape("llama-3.2-3b", 3072, 8192, 28, 24, 8),
    "qwen3-8b": _shape("qwen3-8b", 4096, 12288, 36, 32, 8),
    "llama-3-70b": _shape("llama-3-70b", 8192, 28672, 80, 64, 8),
}

ModelLike = Union[ModelShape, str]


def _model(model: ModelLike) -> ModelShape:
    return MODELS[model] if isinstance(model, str) else model


# Hardware budgets of one B200 SM / CTA.
SMEM_BUDGET_BYTES = 232448   # 227 KB opt-in dynamic shared memory per CTA
TMEM_COLUMNS = 512           # 128 lanes x 512 columns of 32-bit per SM
NUM_SMS_B200 = 148
VMEM_BUDGET_BYTES = SMEM_BUDGET_BYTES

# Stage ids of the library (svdmlp_set_split_override / svdmlp_plan_info).
STAGE_XU, STAGE_GATE_UP, STAGE_DOWN_U, STAGE_DOWN_V = 0, 1, 2, 3


class TileInfo(NamedTuple):
    """Compile-time resources of the kernel one stage runs with (svdmlp_tile_info)."""
    tile_rows: int      # activation rows per tile (256 for CTA pairs; the token tile at decode sizes)
    tile_cols: int      # output features per tile
    tile_k: int         # K per pipeline stage
    stages: int         # pipeline depth
    smem_bytes: int     # dynamic shared memory per CTA
    tmem_columns: int   # tensor-memory columns per CTA
    threads: int        # threads per CTA
    ctas_per_tile: int  # 2 for CTA-pair (cta_group::2) tiles


class Plan(NamedTuple):
    """Work decomposition of one stage launch (svdmlp_plan_info)."""
    m_tiles: int
    n_tiles: int
    k_blocks: int
    splits: int
    units: int
    grid: int


def tile_info(stage: int, rows: int) -> TileInfo:
    out = (ctypes.c_int * 8)()
    _lib.check(_lib.load().svdmlp_tile_info(int(stage), int(rows), out), "tile_info")
    return TileInfo(*list(out))


def stage_plan(stage: int, rows: int, n: int, k: int) -> Plan:
    out = (ctypes.c_int * 6)()
    _lib.check(_lib.load().svdmlp_plan_info(int(stage), int(rows), int(n), int(k), out), "plan_info")
    return Plan(*list(out))


# Down-kernel tile constants under the reference names (the prefill T.v_down /
# H.u_down tiles: 128 rows per CTA, 64-wide K blocks, 256-wide N tiles).
XUV_ROW_TILE = 128
XUV_INPUT_TILE = 64
XUV_RANK_TILE = 256
XUV_OUTPUT_TILE = 256


class GateUpBlocks(NamedTuple):
    """Gate/up tiling: ``bs`` activation rows per tile, ``bh`` K block of
    X.[u_g|u_u] (over hidden), ``br`` K block of the SwiGLU GEMM (over the
    rank), ``bn`` ff columns per branch and tile, and ``splits``, the split-K
    count of the SwiGLU GEMM (0: the library's planner).  Tile shapes are
    compile-time on B200; ``splits`` is applied per call."""
    bs: int
    bh: int
    br: int
    bn: int
    splits: int = 0


def rank_for(model: ModelLike, ratio: float) -> int:
    """128-aligned rank of a model's factors at a compression ratio
    (kernels/reference.py:21-34 applied to the model's shape)."""
    m = _model(model)
    return low_rank_dim(m.hidden_size, m.intermediate_size, ratio)


def benchmark_rank(model: ModelLike, ratio: float) -> int:
    """floor(ratio * in * out / (in + out)): the rank of the benchmark configurations."""
    m = _model(model)
    return rank_for_ratio(m.hidden_size, m.intermediate_size, ratio)


def gate_up_block_params(rows: int, model: ModelLike = "llama-3.1-8b", ratio: float = 0.8) -> GateUpBlocks:
    """The gate/up tiling and split-K plan the B200 kernels use for `rows`
    tokens of `model` at `ratio` (the reference's get_fused_mlp_up_T_params,
    test_speedup.py:169-177)."""
    m = _model(model)
    r = rank_for(m, ratio)
    t_xu = tile_info(STAGE_XU, rows)
    t_gu = tile_info(STAGE_GATE_UP, rows)
    plan = stage_plan(STAGE_GATE_UP, rows, m.intermediate_size, r)
    return GateUpBlocks(bs=t_gu.tile_rows, bh=t_xu.tile_k, br=t_gu.tile_k, bn=t_gu.tile_cols, splits=plan.splits)


def gate_up_tuning_candidates(rows: int, model: ModelLike = "llama-3.1-8b", ratio: float = 0.8, profile=None):
    """Candidates for the gate/up tuner (bench/tune.py:135-137): the compiled
    tile with every split-K count the SwiGLU GEMM can take at this size (at
    least 8 k-blocks per split for CTA pairs, 2 for the decode kernels), the
    planner's choice first.  ``profile`` is accepted for the reference's
    signature; "quick" keeps the planner's choice and its two neighbours."""
    base = gate_up_block_params(rows, model, ratio)
    m = _model(model)
    r = rank_for(m, ratio)
    k_blocks = -(-r // base.br)
    min_kb = 8 if base.bs >= 256 else 2
    feasible = [s for s in range(1, 9) if -(-k_blocks // s) >= min_kb]
    chosen = max(1, base.splits)
    order = [chosen] + [s for s in feasible if s != chosen]
    if profile == "quick":
        order = [s for s in order if abs(s - chosen) <= 1]
    return [base._replace(splits=s) for s in order]


def _pair_smem(bn: int, nb: int, shared_a: bool, stages: int, out_bytes: int, epi_warps: int, ctas: int) -> int:
    """Shared memory of a tcgen05 GEMM tile with this shape, laid out as the
    kernel lays it out (gemm_sm100.cuh GemmCfg): the operand ring, the output
    staging boxes, the barriers and the alignment slack."""
    a = 128 * 64 * 2
    b = (bn // ctas) * 64 * 2
    na = 1 if (nb == 1 or shared_a) else 2
    staging = epi_warps * 2 * 32 * 32 * out_bytes
    bars = (2 * stages + 5) * 8
    return stages * (na * a + nb * b) + staging + bars + 64 + 1024


def smem_bytes_gate_up(blocks: Optional[GateUpBlocks] = None, r_pad: int = 0, hidden: int = 0) -> int:
    """Shared memory per CTA of the gate/up SwiGLU GEMM.  Without `blocks`
    (or with the compiled tile) it is the compiled kernel's; with another
    `bn` it is what that tile would need in the same layout (the budget check
    for a tuner's request)."""
    t = tile_info(STAGE_GATE_UP, 1024)
    if blocks is None or int(blocks.bn) == t.tile_cols:
        return t.smem_bytes
    return _pair_smem(int(blocks.bn), 2, False, t.stages, 2, 8, t.ctas_per_tile)


def tmem_columns_gate_up(blocks: Optional[GateUpBlocks] = None) -> int:
    """TMEM columns of the dual accumulator (gate and up, each rounded up to
    128 or 256 columns)."""
    bn = tile_info(STAGE_GATE_UP, 1024).tile_cols if blocks is None else int(blocks.bn)
    return 2 * (128 if bn <= 128 else 256) if bn <= 256 else 2 * bn


def smem_bytes_xuv(intermediate: int = 0, r_pad: int = 0, hidden: int = 0) -> int:
    """Shared memory per CTA of the down operator's two GEMMs (the larger)."""
    return max(tile_info(STAGE_DOWN_U, 1024).smem_bytes, tile_info(STAGE_DOWN_V, 1024).smem_bytes)


def smem_bytes_gate_up_down_u(blocks=None, r_g: int = 0, r_d: int = 0, hidden: int = 0) -> int:
    return max(smem_bytes_gate_up(blocks), smem_bytes_xuv())


def fits_smem(nbytes: int) -> bool:
    return nbytes <= SMEM_BUDGET_BYTES


def check_budget(nbytes: int, what: str = "kernel", tmem_columns: int = 0) -> None:
    """Raises the reference's budget error (test_speedup.py:303-317) when a
    tile needs more shared memory or tensor memory than a B200 SM has."""
    if not fits_smem(nbytes):
        raise ValueError(f"{what}: SMEM/TMEM budget exceeds {SMEM_BUDGET_BYTES} bytes of shared memory "
                         f"({nbytes} requested)")
    if tmem_columns > TMEM_COLUMNS:
        raise ValueError(f"{what}: SMEM/TMEM budget exceeds {TMEM_COLUMNS} TMEM columns ({tmem_columns} requested)")


def check_gate_up_blocks(blocks: GateUpBlocks) -> None:
    """Validates a gate/up block request the way the reference launcher does
    (positive integers, then the on-chip budget)."""
    for name, value in zip(("bs", "bh", "br", "bn"), tuple(blocks)[:4]):
        if isinstance(value, bool) or int(value) != value or int(value) <= 0:
            raise ValueError(f"{name} must be a positive integer, got {value}")
    splits = tuple(blocks)[4] if len(tuple(blocks)) > 4 else 0
    if int(splits) < 0:
        raise ValueError(f"splits must be a non-negative integer, got {splits}")
    check_budget(smem_bytes_gate_up(blocks), "gate/up", tmem_columns_gate_up(blocks))


vmem_bytes_gate_up = smem_bytes_gate_up
vmem_bytes_xuv = smem_bytes_xuv
vmem_bytes_gate_up_down_u = smem_bytes_gate_up_down_u
fits_vmem = fits_smem
