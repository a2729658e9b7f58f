"""svdflash_tpu.kernels.pallas_ops on B200: the operator names the reference's
benches and model call, backed by the sm_100a kernels (see
svdflash_b200.kernels.ops)."""
from svdflash_b200.kernels.ops import (  # noqa: F401
    contracted_svd_mlp, dense_matmul, dense_mlp, fused_gate_up, svd_mlp, xuv_matmul,
)
