"""svdflash_tpu.kernels.reference on B200 (see svdflash_b200.kernels.reference_api)."""
from svdflash_b200.kernels.reference_api import (  # noqa: F401
    dense_mlp_ref, fused_gate_up_ref, fused_xuv_ref, low_rank_dim, silu, svd_mlp_ref,
)
