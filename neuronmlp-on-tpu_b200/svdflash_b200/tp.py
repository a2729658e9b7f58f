"""Tensor parallelism over the ff dimension of an SVD MLP layer.

Per rank p of P (one process per GPU):
  X.[u_gate|u_up]            replicated            (stage 1)
  v_gate, v_up               column-sharded [r, ff/P] -> H_p [M, ff/P] (stage 2)
  u_down                     row-sharded   [ff/P, r_d] -> partial_p = H_p.u_down_p  fp16 or fp32 (stage 3)
  all_reduce(partial, sum)   the only collective (NCCL over NVLink), fp16 by default
                             (half the bytes; the single-GPU layer rounds T to fp16 too)
  .v_down (+ residual)       replicated            (stage 4)

The reference has no multi-device path (models/README.md:26-27); this is the
ff-sharded layer the benchmark configurations ask for.

mode="split" (chosen by mode="auto" for large layers) also shards the two
replicated stages over M (the all-gather
split): X.[u_g|u_u] on this rank's M/P rows, all-gather XU, stages 2-3 on all
rows of this rank's ff shard, reduce-scatter the fp16 partial by rows,
.v_down on this rank's rows, all-gather y.  Three collectives instead of one,
but X.[u_g|u_u] and .v_down cost 1/P each.

collectives="peer" (chosen by "auto" for groups of up to four GPUs that can
all address each other; "peer" selects it for up to eight) runs the exchanges
with the library's own kernels over NVLink peer memory (svdflash_b200.peer):
the partial, XU and y live in a buffer every rank maps, and each collective is
one kernel of plain stores between GPUs.  In the all-reduce mode the exchange
is fused into the H.u_down GEMM: its epilogue stores each partial tile into
this rank's slot of every rank's buffer as the tile finishes, and a small kernel
sums the slots once the peers' flags arrive (the default for two GPUs;
fused_exchange=True/False forces either).  The
fp16 sums are taken in rank order in fp32 and rounded once, so every rank
gets the same bits.  collectives="nccl" uses torch.distributed (NCCL).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _lib
from .kernels import ops
from .peer import PeerBuffer, layout, peer_access_everywhere


def shard_bounds(ff: int, rank: int, world: int) -> tuple[int, int]:
    if ff % world:
        raise ValueError(f"ff={ff} must divide evenly across {world} ranks")
    step = ff // world
    return rank * step, (rank + 1) * step


def gather_rows_forward(forward, x_rows: torch.Tensor, rank: int, world: int, group=None,
                        residual_rows: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                        returns_rows: bool = False) -> torch.Tensor:
    """Runs `forward(x, residual=...)` on the whole batch when each rank holds
    only its row block: rank p passes rows [p*R, (p+1)*R) of X (and of the
    residual) and receives the same rows of the output.  The row blocks are
    all-gathered first (NVLink under NCCL), so that a serving loop that feeds
    each GPU 1/P of the batch from host memory moves 1/P of the bytes over
    each GPU's host link instead of the whole batch.  With `returns_rows`,
    `forward` already returns only this rank's rows."""
    rows = x_rows.shape[0]
    x = torch.empty((rows * world,) + tuple(x_rows.shape[1:]), dtype=x_rows.dtype, device=x_rows.device)
    dist.all_gather_into_tensor(x, x_rows.contiguous(), group=group)
    res = None
    if residual_rows is not None:
        res = torch.empty_like(x)
        dist.all_gather_into_tensor(res, residual_rows.contiguous(), group=group)
    y = forward(x, residual=res)
    mine = y if returns_rows else y[rank * rows:(rank + 1) * rows]
    if out is None:
        return mine if returns_rows else mine.clone()
    out.copy_(mine)
    return out


class TensorParallelSvdMlp:
    """One ff-sharded SVD MLP layer on this rank's GPU."""

    def __init__(self, u_gate, v_gate, u_up, v_up, u_down, v_down, rank: int, world: int, group=None,
                 reduce_dtype: torch.dtype = torch.float16, mode: str = "auto", collectives: str = "auto",
                 fused_exchange: Optional[bool] = None):
        ff = v_gate.shape[1]
        lo, hi = shard_bounds(ff, rank, world)
        if reduce_dtype not in (torch.float16, torch.float32):
            raise TypeError("reduce_dtype must be torch.float16 or torch.float32 (supported dtypes)")
        if mode not in ("auto", "allreduce", "split"):
            raise ValueError("mode must be 'auto', 'allreduce' or 'split'")
        if mode == "split" and reduce_dtype != torch.float16:
            raise TypeError("the split mode reduces an fp16 partial")
        if collectives not in ("auto", "nccl", "peer"):
            raise ValueError("collectives must be 'auto', 'nccl' or 'peer'")
        if collectives == "peer" and reduce_dtype != torch.float16:
            raise TypeError("the peer collectives reduce an fp16 partial")
        self.rank, self.world, self.group, self.reduce_dtype, self.mode = rank, world, group, reduce_dtype, mode
        self.collectives = collectives
        # all-reduce mode on the peer collectives: the exchange runs inside
        # the H.u_down GEMM (False: a separate all-reduce kernel after it;
        # None: fused for groups of up to FUSED_AUTO_MAX_WORLD, as measured)
        self.fused_exchange = world <= self.FUSED_AUTO_MAX_WORLD if fused_exchange is None else bool(fused_exchange)
        self.layer = ops.pack_svd_layer(u_gate, v_gate[:, lo:hi].contiguous(), u_up, v_up[:, lo:hi].contiguous(),
                                        u_down[lo:hi].contiguous(), v_down)
        self.r_d = u_down.shape[1]
        self._partial: Optional[torch.Tensor] = None
        self._peer: Optional[PeerBuffer] = None
        self._peer_m = 0
        self._t_rows: Optional[torch.Tensor] = None

    # ---------------------------------------------------------- peer memory
    def peer_collectives(self) -> bool:
        """Whether the exchanges run on the library's peer-memory kernels
        (decided once, collectively, on the first call that needs it; that
        call and any call that grows the peer buffer exchange handles over the
        process group, so they must run eagerly, not under graph capture)."""
        if self.world == 1 or self.reduce_dtype != torch.float16 or self.collectives == "nccl":
            return False
        if self.collectives == "auto":
            # measured on 2 and 4 GPUs (level with NCCL at 1024 tokens, ahead at
            # decode sizes); larger groups keep NCCL by default until measured
            use = self.world <= self.PEER_AUTO_MAX_WORLD and peer_access_everywhere(self.group)
            self.collectives = "peer" if use else "nccl"
        return self.collectives == "peer"

    PEER_AUTO_MAX_WORLD = 4
    # measured (8B layer at 1024 tokens, fused vs separate): 2 GPUs 209 vs 221
    # us per layer; 4 GPUs 198 vs 182 (each rank stores its whole partial into
    # three peers from the GEMM epilogue)
    FUSED_AUTO_MAX_WORLD = 2

    def _ensure_peer(self, m: int, d: int) -> PeerBuffer:
        """The peer buffer for m rows (collective when it has to grow):
        partial [m, cols] fp16, the reduction's scratch, XU [m, 2 rp_gu] fp16,
        y [m, d] bf16, and, when the exchange is fused, its slots (two sets of
        one fp16 [m, cols] slot per rank)."""
        if self._peer is not None and self._peer_m >= m:
            return self._peer
        if self._peer is not None:
            self._peer.close()
            self._peer = None
        cols = (self.r_d + 7) // 8 * 8
        n1 = 2 * self.layer.layout.rp_gu
        lib = _lib.load()
        signal = int(lib.svdmlp_peer_signal_bytes())
        scratch = int(lib.svdmlp_peer_scratch_bytes(self.world, m, cols))
        slots = int(lib.svdmlp_peer_slots_bytes(self.world, m, cols)) if self.fused_exchange else 0
        (self._off_part, self._off_scr, self._off_xu, self._off_y, self._off_slots), total = layout(
            [m * cols * 2, scratch, m * n1 * 2, m * d * 2, slots], signal)
        self._cols, self._n1 = cols, n1
        self._peer = PeerBuffer(total, self.rank, self.world, self.group)
        self._peer_m = m
        return self._peer

    def close(self) -> None:
        """Frees the peer buffer (collective: every rank calls it)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None
            self._peer_m = 0

    def check_peer_status(self) -> None:
        """Raises if a peer collective's wait expired or an fp16 sum saturated."""
        if self._peer is not None:
            self._peer.check_status()

    def _partial_buffer(self, m: int, device) -> torch.Tensor:
        align = 4 if self.reduce_dtype == torch.float32 else 8
        cols = (self.r_d + align - 1) // align * align   # 16-byte rows for the TMA store and load
        if self._partial is None or self._partial.shape[0] < m or self._partial.device != device:
            self._partial = torch.zeros((m, cols), dtype=self.reduce_dtype, device=device)
        return self._partial[:m]

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        m = x.shape[0]
        if self.world > 1 and m % self.world == 0 and self._use_split(m, x.shape[1]):
            return self._forward_split(x, residual, out)
        if self.peer_collectives():
            pb = self._ensure_peer(m, x.shape[1])
            part = pb.view(self._off_part, (m, self._cols), torch.float16)
            if self.fused_exchange:
                # H.u_down stores this rank's partial into every rank's slot as
                # its tiles finish; the sum waits only for the peers' flags
                ops.forward_partial_peer_packed(self.layer, x, pb, self._off_slots, self._peer_m, self._cols)
                pb.sum_f16(self._off_slots, self._peer_m, m, self._cols, self._cols, part)
            else:
                ops.forward_partial_packed(self.layer, x, part[:, :self.r_d])
                pb.allreduce_f16(self._off_part, m, self._cols, self._cols, self._off_scr)
            return ops.down_finish_packed(self.layer, part[:, :self.r_d], residual=residual, out=out)
        buf = self._partial_buffer(m, x.device)
        ops.forward_partial_packed(self.layer, x, buf[:, :self.r_d])
        if self.world > 1:
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)
        return ops.down_finish_packed(self.layer, buf[:, :self.r_d], residual=residual, out=out)

    __call__ = forward

    def forward_rows(self, x_rows: torch.Tensor, residual: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The layer for a batch whose rows are spread over the ranks: this
        rank passes its row block of X (rows [rank*R, (rank+1)*R) of the
        batch) and gets the same rows of Y (see gather_rows_forward).  In the
        split mode the final all-gather of y is skipped: this rank's rows are
        the ones its `. v_down` produced."""
        if self.world == 1:
            return self.forward(x_rows, residual=residual, out=out)
        m = x_rows.shape[0] * self.world
        if self._use_split(m, x_rows.shape[1]):
            # The split mode only ever reads this rank's rows of X and of the
            # residual: no all-gather of either, only of XU.
            y_p = self._split_rows(x_rows, residual)
            if out is None:
                return y_p
            out.copy_(y_p)
            return out
        return gather_rows_forward(self.forward, x_rows, self.rank, self.world, self.group, residual, out)

    # "auto": the split pays once the replicated stages outweigh the fixed cost
    # of two more collectives (measured on 2 B200s: 70B layer at 4096 tokens
    # 2491 -> 2198 us; 8B layer at 1024 tokens 215 -> 269 us).
    SPLIT_MIN_ELEMENTS = 16 * 1024 * 1024

    def _use_split(self, m: int, d: int) -> bool:
        if self.mode == "auto":
            return self.reduce_dtype == torch.float16 and m * d > self.SPLIT_MIN_ELEMENTS
        return self.mode == "split"

    def _split_rows(self, x_rows: torch.Tensor, residual_rows: Optional[torch.Tensor]) -> torch.Tensor:
        """The split mode from this rank's row block of X (and of the residual)
        to the same rows of y: X.[u_g|u_u] on the block, all-gather XU, stages
        2-3 of this ff shard on all rows, reduce-scatter the fp16 partial by
        rows, . v_down (+ residual) on the block."""
        rows = x_rows.shape[0]
        m = rows * self.world
        dev = x_rows.device
        n1 = 2 * self.layer.layout.rp_gu
        if self.peer_collectives():
            return self._split_rows_peer(x_rows, residual_rows)
        xu_p = ops.xu_project_packed(self.layer, x_rows)
        xu = torch.empty((m, n1), dtype=torch.float16, device=dev)
        dist.all_gather_into_tensor(xu, xu_p, group=self.group)
        ops.partial_from_xu_packed(self.layer, xu, self._partial_buffer(m, dev)[:, :self.r_d])
        full = self._partial[:m]
        t_p = torch.empty((rows, full.shape[1]), dtype=torch.float16, device=dev)
        dist.reduce_scatter_tensor(t_p, full, op=dist.ReduceOp.SUM, group=self.group)
        return ops.down_finish_packed(self.layer, t_p[:, :self.r_d], residual=residual_rows)

    def _split_rows_peer(self, x_rows: torch.Tensor, residual_rows: Optional[torch.Tensor],
                         y_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """_split_rows over peer memory: XU rows are written into the shared
        buffer and gathered there; the partial is reduce-scattered from it."""
        rows, d = x_rows.shape
        m = rows * self.world
        lo = self.rank * rows
        pb = self._ensure_peer(m, d)
        xu = pb.view(self._off_xu, (m, self._n1), torch.float16)
        ops.xu_project_packed(self.layer, x_rows, out=xu[lo:lo + rows])
        pb.allgather(self._off_xu, m, self._n1 * 2, self._n1 * 2)
        part = pb.view(self._off_part, (m, self._cols), torch.float16)
        ops.partial_from_xu_packed(self.layer, xu, part[:, :self.r_d])
        if self._t_rows is None or self._t_rows.shape[0] < rows or self._t_rows.device != x_rows.device:
            self._t_rows = torch.empty((rows, self._cols), dtype=torch.float16, device=x_rows.device)
        t_p = self._t_rows[:rows]
        pb.reduce_scatter_f16(self._off_part, m, self._cols, self._cols, self._off_scr, t_p)
        return ops.down_finish_packed(self.layer, t_p[:, :self.r_d], residual=residual_rows, out=y_out)

    def _forward_split(self, x: torch.Tensor, residual: Optional[torch.Tensor], out: Optional[torch.Tensor]):
        m, d = x.shape
        rows = m // self.world
        lo, hi = self.rank * rows, (self.rank + 1) * rows
        if self.peer_collectives():
            pb = self._ensure_peer(m, d)
            y_all = pb.view(self._off_y, (m, d), torch.bfloat16)
            self._split_rows_peer(x[lo:hi], None if residual is None else residual[lo:hi], y_out=y_all[lo:hi])
            pb.allgather(self._off_y, m, d * 2, d * 2)
            y = out if out is not None else torch.empty((m, d), dtype=torch.bfloat16, device=x.device)
            y.copy_(y_all)
            return y
        y_p = self._split_rows(x[lo:hi], None if residual is None else residual[lo:hi])
        y = out if out is not None else torch.empty((m, d), dtype=torch.bfloat16, device=x.device)
        dist.all_gather_into_tensor(y, y_p, group=self.group)
        return y
