"""svdflash_tpu.kernels.config on B200 (see svdflash_b200.kernels.config)."""
from svdflash_b200.kernels.config import (  # noqa: F401
    MODELS, NUM_SMS_B200, SMEM_BUDGET_BYTES, TMEM_COLUMNS, VMEM_BUDGET_BYTES, XUV_INPUT_TILE, XUV_OUTPUT_TILE,
    XUV_RANK_TILE, XUV_ROW_TILE, GateUpBlocks, ModelShape, Plan, TileInfo, benchmark_rank, check_budget,
    check_gate_up_blocks, fits_smem, fits_vmem, gate_up_block_params, gate_up_tuning_candidates, rank_for,
    smem_bytes_gate_up, smem_bytes_gate_up_down_u, smem_bytes_xuv, stage_plan, tile_info, tmem_columns_gate_up,
    vmem_bytes_gate_up, vmem_bytes_gate_up_down_u, vmem_bytes_xuv,
)
