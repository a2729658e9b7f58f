"""The launcher names of the reference's test_speedup.py, on the B200 kernels.

``svd_mlp_with_fused_kernel`` keeps the reference's up-before-gate argument
order (test_speedup.py:631-655); ``fused_mlp_up_T`` returns the transposed
``[I, S]`` activation that the reference's TPU kernel produces
(test_speedup.py:522-544) and ``fused_three_mm_XTUV`` consumes it
(test_speedup.py:500-519); ``nki_mm`` and ``nki_baseline`` take PyTorch
``[out, in]`` weights (test_speedup.py:658-678).  The Pallas tiling arguments
(``up_T_params``, ``XTUV_params``, ``async_dma``) are accepted and ignored: the
B200 kernels pick their tiles and split-K factors themselves.

``unfused_low_rank_pallas`` and ``unfused_low_rank`` are the comparison arms
of test_speedup.py:690-736: the same layer as six separate GEMMs with the
SiLU product in between, on this library's plain tcgen05 GEMM
(``svdmlp_gemm``) and on the vendor GEMM (cuBLAS through torch.matmul).
"""
from __future__ import annotations

import torch

from . import ops
from .ops import _positive  # noqa: F401  (test_speedup.py:37-41, imported by bench/e2e_block.py:42-48)


def _plan_params(stage: int, s: int) -> dict:
    from . import config
    _positive("S", s)
    t = config.tile_info(stage, s)
    return dict(tile_rows=t.tile_rows, tile_cols=t.tile_cols, tile_k=t.tile_k, stages=t.stages,
                ctas_per_tile=t.ctas_per_tile)


def get_fused_mlp_up_T_params(S):
    """Tile plan of the gate/up SwiGLU GEMM at S tokens (test_speedup.py:169-177):
    the compiled B200 tile (rows, columns per branch, K block, pipeline depth)."""
    return _plan_params(ops._lib.STAGE_GATE_UP, S)


def get_fused_three_mm_XTUV_params(S):
    """Tile plan of the down operator's first GEMM at S tokens (test_speedup.py:180-191)."""
    return _plan_params(ops._lib.STAGE_DOWN_U, S)


def nki_matmul_fully_optimized_(lhsT, rhs, TILES_IN_BLOCK_M=2, TILES_IN_BLOCK_N=2, TILES_IN_BLOCK_K=4, *,
                                mixed_precision=True, interpret=False):
    """lhsT (K, M), rhs (K, N) -> lhsT^T . rhs (M, N) on the tcgen05 GEMM
    (test_speedup.py:548-615, NKI layout kept); the block counts are checked
    and otherwise left to the library's planner."""
    for name, value in zip(("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N", "TILES_IN_BLOCK_K"),
                           (TILES_IN_BLOCK_M, TILES_IN_BLOCK_N, TILES_IN_BLOCK_K)):
        _positive(name, value)
    if lhsT.shape[0] != rhs.shape[0]:
        raise ValueError("lhsT and rhs must have the same contraction dimension")
    return ops.dense_matmul(lhsT.t(), rhs, mixed_precision=mixed_precision, interpret=interpret)


def _swiglu_bf16(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    # SiLU in fp32 rounded to the activation dtype, times up (test_speedup.py:695)
    return torch.nn.functional.silu(gate.float()).to(gate.dtype) * up


def unfused_low_rank_pallas(x, u_up, v_up, u_gate, v_gate, u_down, v_down, *, mixed_precision=True,
                            interpret=False):
    """Six GEMMs on svdmlp_gemm with the SwiGLU product between them: the
    fused kernels' comparison arm built from the same GEMM kernel
    (test_speedup.py:699-736)."""
    mm = lambda a, b: ops.dense_matmul(a, b, mixed_precision=mixed_precision, interpret=interpret)  # noqa: E731
    gate = mm(mm(x, u_gate), v_gate)
    up = mm(mm(x, u_up), v_up)
    return mm(mm(_swiglu_bf16(gate, up), u_down), v_down)


def unfused_low_rank(x, u_up, v_up, u_gate, v_gate, u_down, v_down):
    """The same six GEMMs on the vendor library (cuBLAS through torch.matmul),
    the counterpart of the XLA arm (test_speedup.py:690-696)."""
    gate = (x @ u_gate) @ v_gate
    up = (x @ u_up) @ v_up
    return (_swiglu_bf16(gate, up) @ u_down) @ v_down


def svd_mlp_with_fused_kernel(x, u_up, v_up, u_gate, v_gate, u_down, v_down, up_T_params=None, XTUV_params=None, *,
                              mixed_precision=True, interpret=False, async_dma=True, down_backend="pallas"):
    if down_backend not in ("pallas", "jax"):
        raise ValueError("down_backend must be 'pallas' or 'jax'")
    return ops.svd_mlp(x, u_gate, v_gate, u_up, v_up, u_down, v_down, mixed_precision=mixed_precision,
                       interpret=interpret)


def fused_mlp_up_T(x, u_gate, v_gate, u_up, v_up, *, mixed_precision=True, interpret=False, async_dma=True,
                   **tile_params):
    """Transposed activation [I, S] = (silu(X.Ug.Vg) * (X.Uu.Vu))^T, as a
    transposed view of the kernel's row-major [S, I] output (no copy;
    fused_three_mm_XTUV reads it back without one either)."""
    return ops.fused_gate_up(x, u_gate, v_gate, u_up, v_up, mixed_precision=mixed_precision,
                             interpret=interpret).t()


def fused_three_mm_XTUV(hidden_t, u_down, v_down, *, mixed_precision=True, interpret=False, async_dma=True,
                        **tile_params):
    """[S, H] = (hidden_t^T . U) . V for a transposed activation [I, S]; a
    transposed view of a row-major [S, I] (fused_mlp_up_T's output) is read in
    place, any other layout is copied once."""
    if hidden_t.shape[0] != u_down.shape[0] or u_down.shape[1] != v_down.shape[0]:
        raise ValueError("hidden, U, V contraction dimensions do not match")
    return ops.xuv_matmul(hidden_t.t(), u_down, v_down, mixed_precision=mixed_precision, interpret=interpret)


def nki_mm(x, up_v_proj, up_u_proj, gate_v_proj, gate_u_proj, down_v_proj, down_u_proj, *, mixed_precision=True,
           interpret=False, up_T_params=None, XTUV_params=None, async_dma=True, down_backend="pallas"):
    """torch.nn.Linear-ordered factors ([out, in])."""
    return svd_mlp_with_fused_kernel(x, up_v_proj.t(), up_u_proj.t(), gate_v_proj.t(), gate_u_proj.t(),
                                     down_v_proj.t(), down_u_proj.t(), up_T_params, XTUV_params,
                                     mixed_precision=mixed_precision, interpret=interpret, async_dma=async_dma,
                                     down_backend=down_backend)


def nki_baseline(x, up_proj, gate_proj, down_proj, *, mixed_precision=True, interpret=False, matmul_params=None):
    """Dense SwiGLU with torch.nn.Linear-ordered weights."""
    return ops.dense_mlp(x, gate_proj.t(), up_proj.t(), down_proj.t(), mixed_precision=mixed_precision,
                         interpret=interpret)
