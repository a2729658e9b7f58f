"""NVLink peer memory for the tensor-parallel layer (one process per GPU).

``PeerBuffer`` allocates one buffer per rank through the library
(``svdmlp_peer_alloc``: device memory whose CUDA IPC handle the other ranks
map), exchanges the handles over the process group and maps the peers'
buffers.  Every rank's buffer has the same layout: the signal area of the
library's collectives, then the matrices the layer exchanges.  The
collectives (``allreduce_f16``, ``reduce_scatter_f16``, ``allgather``) are the
library's own kernels: plain 16-byte stores into the other GPUs' buffers over
NVLink, synchronised by per-CTA flags in the signal areas with bounded waits.
The reference has no multi-device path (models/README.md:26-27).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


class _DeviceMemory:
    """A raw device allocation as seen by torch.as_tensor (no ownership)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def peer_access_everywhere(group=None) -> bool:
    """True when this rank's GPU can address every other visible GPU and every
    rank agrees (a collective over the group)."""
    dev = torch.cuda.current_device()
    ok = all(torch.cuda.can_device_access_peer(dev, j) for j in range(torch.cuda.device_count()) if j != dev)
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=torch.device("cuda", dev))
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


class PeerBuffer:
    """`nbytes` of peer-mapped memory on every rank of `group` (collective)."""

    ALIGN = 256

    def __init__(self, nbytes: int, rank: int, world: int, group=None, device=None):
        if world < 1 or world > 8 or not 0 <= rank < world:
            raise ValueError("PeerBuffer needs 1 <= world <= 8 and 0 <= rank < world")
        self.lib = _lib.load()
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.signal_bytes = int(self.lib.svdmlp_peer_signal_bytes())
        self.nbytes = int(nbytes)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        _lib.check(self.lib.svdmlp_peer_alloc(self.nbytes, ctypes.byref(ptr), handle), "peer_alloc")
        self._own = ptr.value
        self._opened = []
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        every = torch.empty(world * 64, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        handles = every.cpu().reshape(world, 64)
        bases = []
        try:
            for i in range(world):
                if i == rank:
                    bases.append(self._own)
                    continue
                h = (ctypes.c_ubyte * 64)(*handles[i].tolist())
                p = ctypes.c_void_p()
                _lib.check(self.lib.svdmlp_peer_open(h, ctypes.byref(p)), "peer_open")
                self._opened.append(p.value)
                bases.append(p.value)
        except Exception:
            # undo this rank's part; the other ranks fail at their next
            # collective (bounded waits) or at the barrier below
            for q in self._opened:
                self.lib.svdmlp_peer_close(ctypes.c_void_p(q))
            self.lib.svdmlp_peer_free(ctypes.c_void_p(self._own))
            self._opened, self._own = [], None
            raise
        self.bases = (ctypes.c_void_p * world)(*bases)
        # every rank has mapped every buffer before any collective runs
        dist.barrier(group=group, device_ids=[self.device.index])
        self.raw = torch.as_tensor(_DeviceMemory(self._own, self.nbytes), device=self.device)

    def view(self, offset: int, shape, dtype: torch.dtype) -> torch.Tensor:
        """A tensor over this rank's buffer at byte `offset` (row-major `shape`)."""
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        if offset < self.signal_bytes or offset % 16 or offset + nbytes > self.nbytes:
            raise ValueError("view outside the buffer's data area")
        return self.raw[offset:offset + nbytes].view(dtype).view(*shape)

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _check_matrix(self, offset: int, m: int, row_bytes: int, ld_bytes: int) -> None:
        # every rank reads the others' copies of this region: it must lie in the buffer
        if m <= 0 or row_bytes <= 0 or ld_bytes < row_bytes or offset < self.signal_bytes or \
                offset + (m - 1) * ld_bytes + row_bytes > self.nbytes:
            raise ValueError("matrix outside the peer buffer's data area")

    def scratch_bytes(self, m: int, c: int) -> int:
        """Bytes of the scratch region an fp16 [m, c] all-reduce or reduce-scatter needs."""
        return int(self.lib.svdmlp_peer_scratch_bytes(self.world, m, c))

    def _check_scratch(self, offset: int, off_scratch: int, m: int, c: int, ld: int) -> None:
        n = self.scratch_bytes(m, c)
        lo, hi = offset, offset + (m - 1) * 2 * ld + 2 * c
        if off_scratch < self.signal_bytes or off_scratch % 16 or off_scratch + n > self.nbytes or \
                not (off_scratch + n <= lo or off_scratch >= hi):
            raise ValueError("scratch outside the data area or overlapping the matrix")

    def allreduce_f16(self, offset: int, m: int, c: int, ld: int, off_scratch: int) -> None:
        self._check_matrix(offset, m, 2 * c, 2 * ld)
        self._check_scratch(offset, off_scratch, m, c, ld)
        _lib.check(self.lib.svdmlp_peer_allreduce_f16(self.bases, self.world, self.rank, offset, m, c, ld,
                                                      off_scratch, self._stream()), "peer_allreduce")

    def reduce_scatter_f16(self, offset: int, m: int, c: int, ld: int, off_scratch: int,
                           out: torch.Tensor) -> torch.Tensor:
        self._check_matrix(offset, m, 2 * c, 2 * ld)
        self._check_scratch(offset, off_scratch, m, c, ld)
        if out.dtype != torch.float16 or out.stride(1) != 1 or out.device != self.device or \
                out.shape[0] < -(-m // self.world) or out.shape[1] < c:
            raise ValueError("out must be a row-major fp16 [ceil(m / world), >= c] matrix on this GPU")
        _lib.check(self.lib.svdmlp_peer_reduce_scatter_f16(self.bases, self.world, self.rank, offset, m, c, ld,
                                                           off_scratch, out.data_ptr(), out.stride(0),
                                                           self._stream()),
                   "peer_reduce_scatter")
        return out

    def allgather(self, offset: int, m: int, row_bytes: int, ld_bytes: int) -> None:
        self._check_matrix(offset, m, row_bytes, ld_bytes)
        _lib.check(self.lib.svdmlp_peer_allgather(self.bases, self.world, self.rank, offset, m, row_bytes,
                                                  ld_bytes, self._stream()), "peer_allgather")

    # ------------------------------------------------ fused exchange slots
    def slots_bytes(self, slot_rows: int, ld: int) -> int:
        """Bytes of the fused exchange's slots: two sets (alternating calls) of
        one fp16 [slot_rows, ld] slot per rank.  A call of m <= slot_rows rows
        uses the first m rows of each slot."""
        return int(self.lib.svdmlp_peer_slots_bytes(self.world, slot_rows, ld))

    def check_slots(self, off_slots: int, slot_rows: int, m: int, ld: int) -> None:
        n = self.slots_bytes(slot_rows, ld)
        if n <= 0 or not 0 < m <= slot_rows or off_slots < self.signal_bytes or off_slots % 16 or \
                off_slots + n > self.nbytes:
            raise ValueError("exchange slots outside the peer buffer's data area")

    def sum_f16(self, off_slots: int, slot_rows: int, m: int, c: int, ld: int, out: torch.Tensor) -> torch.Tensor:
        """The receiving half of the fused exchange: waits (bounded) until every
        peer has filled its slot for this call, then writes the ranks' fp16
        partials summed in rank order (fp32, rounded once) into `out`, a
        row-major fp16 [m, >= c] matrix on this GPU."""
        self.check_slots(off_slots, slot_rows, m, ld)
        if c <= 0 or c % 8 or c > ld or out.dtype != torch.float16 or out.stride(1) != 1 or \
                out.device != self.device or out.shape[0] < m or out.shape[1] < c:
            raise ValueError("out must be a row-major fp16 [m, >= c] matrix on this GPU (c a multiple of 8)")
        _lib.check(self.lib.svdmlp_peer_sum_f16(self.bases, self.world, self.rank, off_slots, slot_rows, m, c, ld,
                                                out.data_ptr(), out.stride(0), self._stream()), "peer_sum")
        return out

    def check_status(self) -> None:
        """Raises if a collective's wait expired (SvdMlpError) or an fp16 sum
        saturated (SvdMlpRangeError); synchronises the current stream."""
        _lib.check(self.lib.svdmlp_peer_check_status(ctypes.c_void_p(self._own), self._stream()), "peer status")

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this one (collective: every rank
        calls it; no rank frees its buffer while another still maps it)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group, device_ids=[self.device.index])
        self.raw = None
        for p in self._opened:
            self.lib.svdmlp_peer_close(ctypes.c_void_p(p))
        self._opened = []
        dist.barrier(group=self.group, device_ids=[self.device.index])
        self.lib.svdmlp_peer_free(ctypes.c_void_p(self._own))
        self._own = None


def layout(offsets_and_sizes, signal_bytes: int, align: int = PeerBuffer.ALIGN):
    """Byte offsets of consecutive regions after the signal area; returns
    (offsets, total bytes)."""
    offs = []
    cur = signal_bytes
    for size in offsets_and_sizes:
        cur = (cur + align - 1) // align * align
        offs.append(cur)
        cur += int(size)
    return offs, (cur + align - 1) // align * align


__all__ = ["PeerBuffer", "peer_access_everywhere", "layout"]
