"""The launcher names of the reference's test_speedup.py, on the B200 kernels.

``svd_mlp_with_fused_kernel`` keeps the reference's up-before-gate argument
order (test_speedup.py:631-655); ``fused_mlp_up_T`` returns the transposed
``[I, S]`` activation that the reference's TPU kernel produces
(test_speedup.py:522-544) and ``fused_three_mm_XTUV`` consumes it
(test_speedup.py:500-519); ``nki_mm`` and ``nki_baseline`` take PyTorch
``[out, in]`` weights (test_speedup.py:658-678).  The Pallas tiling arguments
(``up_T_params``, ``XTUV_params``, ``async_dma``) are accepted and ignored: the
B200 kernels pick their tiles and split-K factors themselves.
"""
from __future__ import annotations

from . import ops


def svd_mlp_with_fused_kernel(x, u_up, v_up, u_gate, v_gate, u_down, v_down, up_T_params=None, XTUV_params=None, *,
                              mixed_precision=True, interpret=False, async_dma=True, down_backend="pallas"):
    if down_backend not in ("pallas", "jax"):
        raise ValueError("down_backend must be 'pallas' or 'jax'")
    return ops.svd_mlp(x, u_gate, v_gate, u_up, v_up, u_down, v_down, mixed_precision=mixed_precision,
                       interpret=interpret)


def fused_mlp_up_T(x, u_gate, v_gate, u_up, v_up, *, mixed_precision=True, interpret=False, async_dma=True,
                   **tile_params):
    """Transposed activation [I, S] = (silu(X.Ug.Vg) * (X.Uu.Vu))^T."""
    return ops.fused_gate_up(x, u_gate, v_gate, u_up, v_up, mixed_precision=mixed_precision,
                             interpret=interpret).t().contiguous()


def fused_three_mm_XTUV(hidden_t, u_down, v_down, *, mixed_precision=True, interpret=False, async_dma=True,
                        **tile_params):
    """[S, H] = (hidden_t^T . U) . V for a transposed activation [I, S]."""
    if hidden_t.shape[0] != u_down.shape[0] or u_down.shape[1] != v_down.shape[0]:
        raise ValueError("hidden, U, V contraction dimensions do not match")
    return ops.xuv_matmul(hidden_t.t().contiguous(), u_down, v_down, mixed_precision=mixed_precision,
                          interpret=interpret)


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
