"""svdflash_tpu.test_speedup's launcher names on B200 (see
svdflash_b200.kernels.launchers): what bench/e2e_block.py:42-48 imports."""
from svdflash_b200.kernels.launchers import (  # noqa: F401
    _positive, fused_mlp_up_T, fused_three_mm_XTUV, get_fused_mlp_up_T_params, get_fused_three_mm_XTUV_params,
    nki_baseline, nki_matmul_fully_optimized_, nki_mm, svd_mlp_with_fused_kernel, unfused_low_rank,
    unfused_low_rank_pallas,
)
