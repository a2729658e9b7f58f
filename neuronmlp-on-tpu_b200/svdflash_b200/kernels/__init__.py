"""Operator API (mirrors svdflash_tpu.kernels.reference / pallas_ops / config)."""
from . import config, ops  # noqa: F401
from .ops import (  # noqa: F401
    contracted_svd_mlp, dense_matmul, dense_mlp, fused_gate_up, fused_xuv, low_rank_dim, silu, svd_mlp,
    xuv_matmul,
)
