"""Tensor parallelism over the ff dimension of an SVD MLP layer.

Per rank p of P (one process per GPU):
  X.[u_gate|u_up]            replicated            (stage 1)
  v_gate, v_up               column-sharded [r, ff/P] -> H_p [M, ff/P] (stage 2)
  u_down                     row-sharded   [ff/P, r_d] -> partial_p = H_p.u_down_p  fp32 (stage 3)
  all_reduce(partial, sum)   the only collective (NCCL over NVLink), fp16 by default
                             (half the bytes; the single-GPU layer rounds T to fp16 too)
  .v_down (+ residual)       replicated            (stage 4)

The reference has no multi-device path (models/README.md:26-27); this is the
ff-sharded layer the benchmark configurations ask for.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .kernels import ops


def shard_bounds(ff: int, rank: int, world: int) -> tuple[int, int]:
    if ff % world:
        raise ValueError(f"ff={ff} must divide evenly across {world} ranks")
    step = ff // world
    return rank * step, (rank + 1) * step


class TensorParallelSvdMlp:
    """One ff-sharded SVD MLP layer on this rank's GPU."""

    def __init__(self, u_gate, v_gate, u_up, v_up, u_down, v_down, rank: int, world: int, group=None,
                 reduce_dtype: torch.dtype = torch.float16):
        ff = v_gate.shape[1]
        lo, hi = shard_bounds(ff, rank, world)
        if reduce_dtype not in (torch.float16, torch.float32):
            raise TypeError("reduce_dtype must be torch.float16 or torch.float32 (supported dtypes)")
        self.rank, self.world, self.group, self.reduce_dtype = rank, world, group, reduce_dtype
        self.layer = ops.pack_svd_layer(u_gate, v_gate[:, lo:hi].contiguous(), u_up, v_up[:, lo:hi].contiguous(),
                                        u_down[lo:hi].contiguous(), v_down)
        self.r_d = u_down.shape[1]
        self._partial: Optional[torch.Tensor] = None

    def _partial_buffer(self, m: int, device) -> torch.Tensor:
        align = 4 if self.reduce_dtype == torch.float32 else 8
        cols = (self.r_d + align - 1) // align * align   # 16-byte rows for the TMA store and load
        if self._partial is None or self._partial.shape[0] < m or self._partial.device != device:
            self._partial = torch.zeros((m, cols), dtype=self.reduce_dtype, device=device)
        return self._partial[:m]

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        m = x.shape[0]
        buf = self._partial_buffer(m, x.device)
        ops.forward_partial_packed(self.layer, x, buf[:, :self.r_d])
        if self.world > 1:
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)
        return ops.down_finish_packed(self.layer, buf[:, :self.r_d], residual=residual, out=out)

    __call__ = forward
