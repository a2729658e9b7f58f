"""The operator API of the reference's kernels/reference.py, computed on B200.

Same names, argument order and layouts as kernels/reference.py:21-106
(``low_rank_dim``, ``silu``, ``fused_gate_up_ref``, ``fused_xuv_ref``,
``svd_mlp_ref``, ``dense_mlp_ref``): NumPy arrays in, NumPy arrays out in
``x.dtype`` (torch tensors are accepted too and returned as tensors).  The
arrays are moved to the current CUDA device and run through the sm_100a
kernels (svdflash_b200.kernels.ops); there is no host computation path.

Precision differs from the reference's fp32 NumPy by design: fp32 inputs are
rounded to bf16 and the kernels accumulate in fp32 with fp16 intermediates,
which stays within the north-star tolerance of the fp32 result (relative
Frobenius error <= 5e-3, max-abs <= 2e-2 x RMS).
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops

__all__ = ["low_rank_dim", "silu", "fused_gate_up_ref", "fused_xuv_ref", "svd_mlp_ref", "dense_mlp_ref"]

low_rank_dim = ops.low_rank_dim


def _device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("the B200 operators need a CUDA device (there is no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


def _in(a, device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device)
    arr = np.ascontiguousarray(a)
    if arr.dtype.name == "bfloat16":          # ml_dtypes.bfloat16 arrays
        return torch.from_numpy(arr.view(np.uint16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(arr.astype(np.float32, copy=False)).to(device)


def _out(y: torch.Tensor, like):
    if isinstance(like, torch.Tensor):
        return y.to(like.dtype)
    host = y.float().cpu().numpy()
    dtype = np.asarray(like).dtype
    if dtype.name == "bfloat16":
        return host.astype(dtype)
    return host.astype(dtype, copy=False)


def _run(fn, x, *arrays):
    dev = _device()
    xt = _in(x, dev)
    ts = [_in(a, dev) for a in arrays]
    if xt.dtype != torch.bfloat16:
        xt = xt.to(torch.float32)
        ts = [t.to(torch.float32) for t in ts]
    else:
        ts = [t.to(torch.bfloat16) for t in ts]
    return _out(fn(xt, *ts), x)


def silu(x):
    """fp32 x * sigmoid(x) (kernels/reference.py:37-51), on the device."""
    dev = _device()
    y = ops.silu(_in(x, dev))
    return y if isinstance(x, torch.Tensor) else y.cpu().numpy()


def fused_gate_up_ref(x, u_gate, v_gate, u_up, v_up):
    """silu((x.u_gate).v_gate) * ((x.u_up).v_up) (kernels/reference.py:54-72)."""
    return _run(ops.fused_gate_up, x, u_gate, v_gate, u_up, v_up)


def fused_xuv_ref(x, u, v):
    """(x.u).v (kernels/reference.py:75-82)."""
    return _run(ops.xuv_matmul, x, u, v)


def svd_mlp_ref(x, u_gate, v_gate, u_up, v_up, u_down, v_down):
    """fused_xuv_ref(fused_gate_up_ref(x)) as one layer (kernels/reference.py:85-93)."""
    return _run(ops.svd_mlp, x, u_gate, v_gate, u_up, v_up, u_down, v_down)


def dense_mlp_ref(x, w_gate, w_up, w_down):
    """Dense SwiGLU (kernels/reference.py:96-106)."""
    return _run(ops.dense_mlp, x, w_gate, w_up, w_down)
