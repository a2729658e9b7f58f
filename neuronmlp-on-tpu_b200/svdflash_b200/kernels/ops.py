"""B200 operator API of the SVD-compressed SwiGLU MLP.

Two reference interfaces are mirrored here, both backed only by the sm_100a
library (``libsvdmlp.so`` through ``include/svdmlp.h``):

* the golden operator names of ``kernels/reference.py`` (``low_rank_dim``,
  ``silu``, ``fused_gate_up``, ``fused_xuv``, ``svd_mlp``, ``dense_mlp``), with
  the same argument order and natural ``[S, H]`` / ``[S, I]`` layouts;
* the ``pallas_ops`` names the reference benches and model call
  (``svd_mlp``, ``contracted_svd_mlp``, ``fused_gate_up``, ``xuv_matmul``,
  ``dense_mlp``, ``dense_matmul``), with the same keyword arguments
  (call sites: bench/latency.py:346-418, bench/smoke.py:81-83,
  bench/speedup.py:142-143, models/modeling_llama.py:851-937).

Inputs are CUDA tensors.  bf16 inputs compute in bf16 with fp32 accumulation
(the intermediates of the SVD layer are kept in fp16, see include/svdmlp.h);
fp32 inputs with ``mixed_precision=True`` are rounded to bf16 first, as the
reference's ``_dot`` does (test_speedup.py:63-68), and the result is returned
in ``x.dtype``.  There is no CPU path: ``interpret=True`` and
``mixed_precision=False`` raise.

Validation follows the reference launchers (test_speedup.py:37-49,
500-544): ``ValueError`` for non-2-D/empty inputs and mismatched
contraction or gate/up shapes, ``TypeError`` for mixed or unsupported
dtypes.
"""
from __future__ import annotations

import ctypes
import threading
import weakref
from collections import OrderedDict
from typing import Optional

import torch

from .. import _lib

__all__ = [
    "PackedLayer", "pack_svd_layer", "pack_dense_layer", "low_rank_dim", "rank_for_ratio", "silu",
    "fused_gate_up", "fused_xuv", "xuv_matmul", "svd_mlp", "contracted_svd_mlp", "dense_mlp",
    "dense_matmul", "svd_mlp_packed", "contracted_mlp_packed", "dense_mlp_packed", "gate_up_packed", "xuv_packed",
    "forward_partial_packed", "forward_partial_peer_packed", "down_partial_packed", "down_finish_packed", "rmsnorm", "row_sumsq",
    "svd_block_packed", "workspace_for",
    "check_device_status", "launch_count",
]


# --------------------------------------------------------------------- ranks
def low_rank_dim(hidden_size: int, intermediate_size: int, compress_ratio: float) -> int:
    """Rank used by the reference, rounded to a multiple of 128
    (kernels/reference.py:21-34)."""
    numer = intermediate_size * hidden_size * compress_ratio
    denom = (intermediate_size + hidden_size) * 128
    return round(numer / denom) * 128


def rank_for_ratio(in_features: int, out_features: int, ratio: float) -> int:
    """Rank of the benchmark configurations: floor(ratio * in * out / (in + out))."""
    return int(ratio * in_features * out_features // (in_features + out_features))


def silu(x: torch.Tensor) -> torch.Tensor:
    """fp32 SiLU, as kernels/reference.py:37-51 (a helper, not a hot-path op)."""
    x32 = x.float()
    return x32 * torch.sigmoid(x32)


# ---------------------------------------------------------------- validation
_SUPPORTED = (torch.bfloat16, torch.float32)


def _positive(name, value):
    if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
        raise ValueError(f"{name} must be a positive integer, got {value}")


def _validate_arrays(*arrays: torch.Tensor) -> None:
    for a in arrays:
        if not isinstance(a, torch.Tensor):
            raise TypeError(f"expected a torch.Tensor, got {type(a).__name__}")
        if a.dim() != 2 or min(a.shape) <= 0:
            raise ValueError(f"expected a nonempty 2D array, got {tuple(a.shape)}")
        if a.dtype != arrays[0].dtype:
            raise TypeError("all inputs must have the same dtype")
    if arrays[0].dtype not in _SUPPORTED:
        raise TypeError("supported dtypes are bfloat16 and float32")
    dev = arrays[0].device
    for a in arrays:
        if a.device.type != "cuda" or a.device != dev:
            raise ValueError("inputs must be CUDA tensors on one device (the B200 path has no CPU fallback)")


def _check_modes(mixed_precision: bool, interpret: bool, dtype: torch.dtype) -> None:
    if interpret:
        raise NotImplementedError("interpret mode runs Pallas on the CPU; the B200 path has no CPU fallback")
    if not mixed_precision and dtype == torch.float32:
        raise NotImplementedError(
            "fp32 arithmetic (mixed_precision=False) is not provided by the B200 kernels; "
            "they compute in bf16/fp16 with fp32 accumulation")


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


def _ld(t: torch.Tensor) -> int:
    if t.stride(1) != 1:
        raise ValueError("matrices must be row-major (unit column stride)")
    return t.stride(0)


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


# ----------------------------------------------------------------- workspace
_ws_lock = threading.Lock()
_ws_pool: dict = {}


class _Workspace:
    def __init__(self, device: torch.device, nbytes: int):
        self.tensor = torch.empty(int(nbytes), dtype=torch.uint8, device=device)
        self.nbytes = int(nbytes)
        _lib.check(_lib.load().svdmlp_workspace_init(self.ptr, self.nbytes, _stream(device)), "workspace_init")

    @property
    def ptr(self) -> int:
        return self.tensor.data_ptr()


def workspace_for(device: torch.device, nbytes: int) -> _Workspace:
    """Per-(device, stream) workspace, grown on demand and then reused."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    with _ws_lock:
        ws = _ws_pool.get(key)
        if ws is None or ws.nbytes < nbytes:
            if ws is not None:
                torch.cuda.current_stream(device).synchronize()
            ws = _Workspace(device, max(int(nbytes), 1 << 20))
            _ws_pool[key] = ws
    return ws


def check_device_status(device: Optional[torch.device] = None) -> None:
    """Synchronises and raises if a bounded device wait expired (SvdMlpError) or
    an fp16 intermediate saturated (SvdMlpRangeError) on any pooled workspace
    since the last check."""
    lib = _lib.load()
    with _ws_lock:
        items = list(_ws_pool.items())
    for (dev_index, stream), ws in items:
        if device is not None and device.index != dev_index:
            continue
        _lib.check(lib.svdmlp_check_device_status(ws.ptr, ws.nbytes, ctypes.c_void_p(stream)), "device status")


def launch_count() -> int:
    """Kernel launches the library has enqueued since it was loaded."""
    return int(_lib.load().svdmlp_launch_count())


# ------------------------------------------------------------- packed layers
class PackedLayer:
    """Packed (K-major, TMA-legal) weights of one MLP layer on one device."""

    def __init__(self, layout: _lib.Layout, packed: torch.Tensor):
        self.layout = layout
        self.packed = packed

    kind = property(lambda self: self.layout.kind)
    d = property(lambda self: self.layout.d)
    ff = property(lambda self: self.layout.ff)
    r_gu = property(lambda self: self.layout.r_gu)
    r_d = property(lambda self: self.layout.r_d)
    device = property(lambda self: self.packed.device)

    def workspace(self, m: int) -> _Workspace:
        need = _lib.load().svdmlp_workspace_bytes(ctypes.byref(self.layout), int(m))
        if need < 0:
            _lib.check(int(need), "workspace_bytes")
        return workspace_for(self.packed.device, need)

    @property
    def nbytes(self) -> int:
        return int(self.layout.packed_bytes)


def pack_svd_layer(u_gate=None, v_gate=None, u_up=None, v_up=None, u_down=None, v_down=None,
                   norm_weight=None) -> PackedLayer:
    """Packs factor pairs in the reference layouts (u [in, r], v [r, out]).

    Either half may be omitted (gate/up-only or down-only layers).  With
    `norm_weight` ([d]) the layer is packed for svd_block_packed: the decoder
    block's RMSNorm weight is folded into u_gate and u_up."""
    have_gu = u_gate is not None
    have_d = u_down is not None
    if not have_gu and not have_d:
        raise ValueError("at least one factor pair is required")
    arrays = [a for a in (u_gate, v_gate, u_up, v_up, u_down, v_down) if a is not None]
    _validate_arrays(*arrays)
    d = ff = None
    r_gu = r_d = 0
    if have_gu:
        if v_gate is None or u_up is None or v_up is None:
            raise ValueError("gate/up need u_gate, v_gate, u_up and v_up")
        if tuple(u_gate.shape) != tuple(u_up.shape) or tuple(v_gate.shape) != tuple(v_up.shape):
            raise ValueError("gate and up factors must have matching shapes")
        if u_gate.shape[1] != v_gate.shape[0]:
            raise ValueError("u_gate/v_gate contraction dimensions do not match")
        d, r_gu, ff = u_gate.shape[0], u_gate.shape[1], v_gate.shape[1]
    if have_d:
        if v_down is None:
            raise ValueError("down needs u_down and v_down")
        if u_down.shape[1] != v_down.shape[0]:
            raise ValueError("u_down/v_down contraction dimensions do not match")
        if have_gu and (u_down.shape[0] != ff or v_down.shape[1] != d):
            raise ValueError("down factors do not match the gate/up dimensions")
        ff, r_d, d = u_down.shape[0], u_down.shape[1], v_down.shape[1]
    lib = _lib.load()
    layout = _lib.Layout()
    _lib.check(lib.svdmlp_layout_init(ctypes.byref(layout), d, ff, r_gu, r_d), "layout_init")
    dev = arrays[0].device
    packed = torch.empty(int(layout.packed_bytes), dtype=torch.uint8, device=dev)
    bf = [None if a is None else _bf16(a).contiguous() for a in (u_gate, v_gate, u_up, v_up, u_down, v_down)]
    args = []
    for a in bf:
        args += [_ptr(a), 0 if a is None else _ld(a)]
    if norm_weight is not None:
        if not (have_gu and have_d):
            raise ValueError("a block's norm needs a full SVD layer")
        nw = _bf16(norm_weight).reshape(-1).contiguous()
        if nw.numel() != d or nw.device != dev:
            raise ValueError("norm_weight must be [d] on the factors' device: dimensions do not match")
        _lib.check(lib.svdmlp_pack_block(ctypes.byref(layout), nw.data_ptr(), *args, packed.data_ptr(),
                                         _stream(dev)), "pack_block")
    else:
        _lib.check(lib.svdmlp_pack(ctypes.byref(layout), *args, packed.data_ptr(), _stream(dev)), "pack")
    # packing is a set-up step: synchronise once to refuse weights fp16 cannot hold
    _lib.check(lib.svdmlp_pack_status(ctypes.byref(layout), packed.data_ptr(), _stream(dev)), "pack")
    layer = PackedLayer(layout, packed)
    layer.normed = norm_weight is not None
    return layer


def pack_dense_layer(w_gate, w_up, w_down) -> PackedLayer:
    """Packs dense SwiGLU weights w_gate, w_up [H, I] and w_down [I, H]."""
    _validate_arrays(w_gate, w_up, w_down)
    if tuple(w_gate.shape) != tuple(w_up.shape):
        raise ValueError("gate and up weights must have matching shapes")
    d, ff = w_gate.shape
    if tuple(w_down.shape) != (ff, d):
        raise ValueError("w_down dimensions do not match")
    lib = _lib.load()
    layout = _lib.Layout()
    _lib.check(lib.svdmlp_dense_layout_init(ctypes.byref(layout), d, ff), "dense_layout_init")
    dev = w_gate.device
    packed = torch.empty(int(layout.packed_bytes), dtype=torch.uint8, device=dev)
    wg, wu, wd = (_bf16(a).contiguous() for a in (w_gate, w_up, w_down))
    _lib.check(lib.svdmlp_dense_pack(ctypes.byref(layout), wg.data_ptr(), _ld(wg), wu.data_ptr(), _ld(wu),
                                     wd.data_ptr(), _ld(wd), packed.data_ptr(), _stream(dev)), "dense_pack")
    _lib.check(lib.svdmlp_pack_status(ctypes.byref(layout), packed.data_ptr(), _stream(dev)), "dense_pack")
    return PackedLayer(layout, packed)


# Packed-weight cache for the factor-taking API: keyed on the factor tensors'
# identity, storage address and version counter; an entry is dropped when any
# of its tensors is garbage-collected or modified in place.
class _PackCache:
    def __init__(self, capacity: int = 256):
        self.capacity = capacity
        self.entries: OrderedDict = OrderedDict()
        self.lock = threading.Lock()

    @staticmethod
    def _sig(tensors):
        return tuple((id(t), t.data_ptr(), t._version, tuple(t.shape), tuple(t.stride()), t.dtype)
                     for t in tensors)

    def get(self, tag, tensors, build):
        key = (tag,) + self._sig(tensors)
        with self.lock:
            hit = self.entries.get(key)
            if hit is not None:
                refs, layer = hit
                if all(r() is t for r, t in zip(refs, tensors)):
                    self.entries.move_to_end(key)
                    return layer
                del self.entries[key]
        layer = build()
        with self.lock:
            self.entries[key] = ([weakref.ref(t) for t in tensors], layer)
            while len(self.entries) > self.capacity:
                self.entries.popitem(last=False)
        return layer

    def clear(self):
        with self.lock:
            self.entries.clear()


_cache = _PackCache()


def clear_pack_cache() -> None:
    _cache.clear()


# ----------------------------------------------------------- packed entries
def _prep_x(x: torch.Tensor, d: int):
    xb = _bf16(x)
    if xb.stride(1) != 1:
        xb = xb.contiguous()
    if xb.shape[1] != d:
        raise ValueError(f"x has {xb.shape[1]} features but the layer expects {d}: dimensions do not match")
    return xb


def _out(m: int, n: int, device) -> torch.Tensor:
    return torch.empty((m, n), dtype=torch.bfloat16, device=device)


def svd_mlp_packed(layer: PackedLayer, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = (silu(x.u_g.v_g) * (x.u_u.v_u)).u_d.v_d (+ residual), bf16 [M, d]."""
    if layer.kind != _lib.KIND_SVD or layer.r_gu == 0 or layer.r_d == 0:
        raise ValueError("svd_mlp needs a full SVD layer")
    xb = _prep_x(x, layer.d)
    m = xb.shape[0]
    y = out if out is not None else _out(m, layer.d, xb.device)
    ws = layer.workspace(m)
    res = None
    if residual is not None:
        res = _bf16(residual)
        if tuple(res.shape) != (m, layer.d):
            raise ValueError("residual shape does not match the output")
    _lib.check(_lib.load().svdmlp_forward(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), xb.data_ptr(), _ld(xb), m, y.data_ptr(), _ld(y),
        _ptr(res), 0 if res is None else _ld(res), ws.ptr, ws.nbytes, _stream(xb.device)), "svd_mlp")
    return y


def row_sumsq(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per row of x [M, d], the sum of squares of each 128-column slice, fp32
    [M, ceil(d / 128)]: the statistics the first block of a stack reads."""
    xb = _bf16(x)
    if xb.stride(1) != 1:
        xb = xb.contiguous()
    m, d = xb.shape
    parts = -(-d // 128)
    if out is None:
        out = torch.empty((m, parts), dtype=torch.float32, device=xb.device)
    if out.dtype != torch.float32 or out.shape[0] < m or out.shape[1] < parts or out.stride(1) != 1:
        raise ValueError("stats must be fp32 [M, ceil(d / 128)]")
    _lib.check(_lib.load().svdmlp_row_sumsq(xb.data_ptr(), _ld(xb), m, d, out.data_ptr(), out.stride(0),
                                            _stream(xb.device)), "row_sumsq")
    return out


def svd_block_packed(layer: PackedLayer, x: torch.Tensor, x_stats: torch.Tensor,
                     y_stats: Optional[torch.Tensor] = None, eps: float = 1e-5,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One decoder-stack block y = x + mlp(rmsnorm(x)) with the norm fused
    (svdmlp_forward_block): `layer` packed with its norm weight, `x_stats` the
    per-slice sums of squares of x (row_sumsq, or the previous block's
    y_stats); y_stats, when given, receives the same statistics of y."""
    if not getattr(layer, "normed", False):
        raise ValueError("svd_block_packed needs a layer packed with norm_weight")
    xb = _prep_x(x, layer.d)
    m = xb.shape[0]
    y = out if out is not None else _out(m, layer.d, xb.device)
    for st in (x_stats, y_stats):
        if st is not None and (st.dtype != torch.float32 or st.stride(1) != 1 or st.shape[0] < m):
            raise ValueError("block statistics must be fp32 [M, ceil(d / 128)] row-major")
    if y_stats is not None and y_stats.stride(0) != x_stats.stride(0):
        raise ValueError("x_stats and y_stats must share their row stride")
    ws = layer.workspace(m)
    _lib.check(_lib.load().svdmlp_forward_block(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), xb.data_ptr(), _ld(xb), m, y.data_ptr(), _ld(y),
        x_stats.data_ptr(), x_stats.stride(0), _ptr(y_stats), float(eps), ws.ptr, ws.nbytes,
        _stream(xb.device)), "svd_block")
    return y


def contracted_mlp_packed(layer: PackedLayer, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The contracted layer (svdmlp_forward_contracted): gate/up fused through
    . u_down at decode sizes, H never written; the two-operator path above 16
    tokens."""
    if layer.kind != _lib.KIND_SVD or layer.r_gu == 0 or layer.r_d == 0:
        raise ValueError("contracted_svd_mlp needs a full SVD layer")
    xb = _prep_x(x, layer.d)
    m = xb.shape[0]
    y = out if out is not None else _out(m, layer.d, xb.device)
    ws = layer.workspace(m)
    res = None
    if residual is not None:
        res = _bf16(residual)
        if tuple(res.shape) != (m, layer.d):
            raise ValueError("residual shape does not match the output")
    _lib.check(_lib.load().svdmlp_forward_contracted(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), xb.data_ptr(), _ld(xb), m, y.data_ptr(), _ld(y),
        _ptr(res), 0 if res is None else _ld(res), ws.ptr, ws.nbytes, _stream(xb.device)), "contracted_svd_mlp")
    return y


def dense_mlp_packed(layer: PackedLayer, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if layer.kind != _lib.KIND_DENSE:
        raise ValueError("dense_mlp needs a dense layer")
    xb = _prep_x(x, layer.d)
    m = xb.shape[0]
    y = out if out is not None else _out(m, layer.d, xb.device)
    ws = layer.workspace(m)
    res = None if residual is None else _bf16(residual)
    _lib.check(_lib.load().svdmlp_dense_forward(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), xb.data_ptr(), _ld(xb), m, y.data_ptr(), _ld(y),
        _ptr(res), 0 if res is None else _ld(res), ws.ptr, ws.nbytes, _stream(xb.device)), "dense_mlp")
    return y


def gate_up_packed(layer: PackedLayer, x: torch.Tensor) -> torch.Tensor:
    if layer.kind != _lib.KIND_SVD or layer.r_gu == 0:
        raise ValueError("fused_gate_up needs gate/up factors")
    xb = _prep_x(x, layer.d)
    m = xb.shape[0]
    h = _out(m, layer.ff, xb.device)
    ws = layer.workspace(m)
    _lib.check(_lib.load().svdmlp_gate_up(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), xb.data_ptr(), _ld(xb), m, h.data_ptr(), _ld(h),
        ws.ptr, ws.nbytes, _stream(xb.device)), "fused_gate_up")
    return h


def xuv_packed(layer: PackedLayer, h: torch.Tensor) -> torch.Tensor:
    if layer.kind != _lib.KIND_SVD or layer.r_d == 0:
        raise ValueError("xuv needs down factors")
    hb = _prep_x(h, layer.ff)
    m = hb.shape[0]
    y = _out(m, layer.d, hb.device)
    ws = layer.workspace(m)
    _lib.check(_lib.load().svdmlp_xuv(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), hb.data_ptr(), _ld(hb), m, y.data_ptr(), _ld(y),
        ws.ptr, ws.nbytes, _stream(hb.device)), "xuv_matmul")
    return y


def forward_partial_packed(layer: PackedLayer, x: torch.Tensor, partial: Optional[torch.Tensor] = None,
                           dtype: torch.dtype = torch.float32):
    """Stages 1-3 of an ff-shard: the [M, r_d] partial for the all-reduce, fp32
    or fp16 (the dtype of `partial` when given, else `dtype`)."""
    xb = _prep_x(x, layer.d)
    m = xb.shape[0]
    if partial is None:
        align = 4 if dtype == torch.float32 else 8
        partial = torch.empty((m, layer.r_d + (-layer.r_d) % align), dtype=dtype, device=xb.device)[:, :layer.r_d]
    if partial.dtype not in (torch.float32, torch.float16):
        raise TypeError("the partial must be fp32 or fp16 (supported dtypes)")
    fn = _lib.load().svdmlp_forward_partial if partial.dtype == torch.float32 else _lib.load().svdmlp_forward_partial_f16
    ws = layer.workspace(m)
    _lib.check(fn(ctypes.byref(layer.layout), layer.packed.data_ptr(), xb.data_ptr(), _ld(xb), m, partial.data_ptr(),
                  partial.stride(0), ws.ptr, ws.nbytes, _stream(xb.device)), "forward_partial")
    return partial


def forward_partial_peer_packed(layer: PackedLayer, x: torch.Tensor, peer, off_slots: int, slot_rows: int,
                                ld_slot: int) -> None:
    """Stages 1-3 of an ff-shard with the exchange fused in: this rank's fp16
    [M, r_d] partial goes straight into its slot of every rank's peer buffer
    (`peer`: a svdflash_b200.peer.PeerBuffer; slots of `slot_rows` rows at
    byte offset `off_slots`, row stride `ld_slot` elements), written by the
    H.u_down GEMM's epilogue at prefill sizes; PeerBuffer.sum_f16 then sums
    them."""
    if layer.kind != _lib.KIND_SVD or layer.r_d == 0:
        raise ValueError("the fused exchange needs an SVD layer")
    xb = _prep_x(x, layer.d)
    m = xb.shape[0]
    if ld_slot < layer.r_d:
        raise ValueError("slot rows must hold r_d columns")
    peer.check_slots(off_slots, slot_rows, m, ld_slot)
    ws = layer.workspace(m)
    _lib.check(_lib.load().svdmlp_forward_partial_f16_peer(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), xb.data_ptr(), _ld(xb), m, peer.bases, peer.world,
        peer.rank, off_slots, slot_rows, ld_slot, ws.ptr, ws.nbytes, _stream(xb.device)), "forward_partial_peer")


def down_partial_packed(layer: PackedLayer, h: torch.Tensor, partial: Optional[torch.Tensor] = None):
    """First half of the down operator on an ff-shard: the fp32 [M, r_d]
    partial h . u_down (h: bf16 [M, ff_shard]), the rank-local term that the
    tensor-parallel layer all-reduces before down_finish_packed."""
    if layer.kind != _lib.KIND_SVD or layer.r_d == 0:
        raise ValueError("down_partial needs down factors")
    hb = _prep_x(h, layer.ff)
    m = hb.shape[0]
    if partial is None:
        partial = torch.empty((m, layer.r_d + (-layer.r_d) % 4), dtype=torch.float32,
                              device=hb.device)[:, :layer.r_d]
    if partial.dtype != torch.float32:
        raise TypeError("the partial must be fp32 (supported dtypes)")
    ws = layer.workspace(m)
    _lib.check(_lib.load().svdmlp_down_partial(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), hb.data_ptr(), _ld(hb), m, partial.data_ptr(),
        partial.stride(0), ws.ptr, ws.nbytes, _stream(hb.device)), "down_partial")
    return partial


def xu_project_packed(layer: PackedLayer, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Stage 1 alone: XU = x . [u_g|u_u], fp16 [M, 2*rp_gu] (the layout stages 2-3 read)."""
    xb = _prep_x(x, layer.d)
    m = xb.shape[0]
    n1 = 2 * layer.layout.rp_gu
    xu = out if out is not None else torch.empty((m, n1), dtype=torch.float16, device=xb.device)
    if xu.dtype != torch.float16 or xu.shape[1] < n1:
        raise ValueError("xu must be fp16 [M, 2*rp_gu]")
    ws = layer.workspace(m)
    _lib.check(_lib.load().svdmlp_xu_project(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), xb.data_ptr(), _ld(xb), m, xu.data_ptr(), _ld(xu),
        ws.ptr, ws.nbytes, _stream(xb.device)), "xu_project")
    return xu


def partial_from_xu_packed(layer: PackedLayer, xu: torch.Tensor, partial: Optional[torch.Tensor] = None):
    """Stages 2-3 of an ff-shard from a given XU: fp16 [M, r_d] partial."""
    m = xu.shape[0]
    if partial is None:
        partial = torch.empty((m, layer.r_d + (-layer.r_d) % 8), dtype=torch.float16, device=xu.device)[:, :layer.r_d]
    if xu.dtype != torch.float16 or partial.dtype != torch.float16:
        raise TypeError("xu and the partial must be fp16 (supported dtypes)")
    ws = layer.workspace(m)
    _lib.check(_lib.load().svdmlp_partial_from_xu_f16(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), xu.data_ptr(), _ld(xu), m, partial.data_ptr(),
        partial.stride(0), ws.ptr, ws.nbytes, _stream(xu.device)), "partial_from_xu")
    return partial


def down_finish_packed(layer: PackedLayer, partial: torch.Tensor, residual: Optional[torch.Tensor] = None,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = sum(partials) . v_down (+ residual) from the all-reduced fp32 or fp16 partial."""
    m = partial.shape[0]
    if partial.dtype not in (torch.float32, torch.float16):
        raise TypeError("the partial must be fp32 or fp16 (supported dtypes)")
    y = out if out is not None else _out(m, layer.d, partial.device)
    ws = layer.workspace(m)
    res = None if residual is None else _bf16(residual)
    fn = _lib.load().svdmlp_down_finish if partial.dtype == torch.float32 else _lib.load().svdmlp_down_finish_f16
    _lib.check(fn(
        ctypes.byref(layer.layout), layer.packed.data_ptr(), partial.data_ptr(), partial.stride(0), m,
        y.data_ptr(), _ld(y), _ptr(res), 0 if res is None else _ld(res), ws.ptr, ws.nbytes,
        _stream(partial.device)), "down_finish")
    return y


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5, out: Optional[torch.Tensor] = None):
    """RMSNorm over the last dim (models/modeling_llama.py:245-262), bf16 in/out."""
    xb = _bf16(x)
    if xb.stride(1) != 1:
        xb = xb.contiguous()
    wb = _bf16(weight).contiguous()
    y = out if out is not None else torch.empty_like(xb)
    _lib.check(_lib.load().svdmlp_rmsnorm(xb.data_ptr(), _ld(xb), wb.data_ptr(), y.data_ptr(), _ld(y),
                                          xb.shape[0], xb.shape[1], float(eps), _stream(xb.device)), "rmsnorm")
    return y


# --------------------------------------------- reference-named entry points
def _finish(y: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    return y if x.dtype == torch.bfloat16 else y.to(x.dtype)


class _GateUpSplits:
    """Applies a block request's split-K count to the SwiGLU GEMM (stage 1)
    for the duration of one call; tile shapes are compile-time on B200."""

    _lock = threading.Lock()

    def __init__(self, blocks):
        self.splits = 0
        if blocks is not None:
            from . import config
            blocks = tuple(blocks)
            config.check_gate_up_blocks(config.GateUpBlocks(*blocks))
            self.splits = int(blocks[4]) if len(blocks) > 4 else 0

    def __enter__(self):
        if self.splits:
            self._lock.acquire()
            _lib.check(_lib.load().svdmlp_set_split_override(_lib.STAGE_GATE_UP, self.splits), "split override")
        return self

    def __exit__(self, *exc):
        if self.splits:
            _lib.load().svdmlp_set_split_override(_lib.STAGE_GATE_UP, 0)
            self._lock.release()
        return False


def fused_gate_up(x, u_gate, v_gate, u_up, v_up, *, blocks=None, mixed_precision=True, interpret=False):
    """[S, I] = silu(X.Ug.Vg) * (X.Uu.Vu) (kernels/reference.py:54-72;
    pallas_ops.fused_gate_up, bench/smoke.py:81-83).  `blocks` (a
    config.GateUpBlocks) is checked against the on-chip budget; its `splits`
    sets the SwiGLU GEMM's split-K count for this call."""
    _validate_arrays(x, u_gate, v_gate, u_up, v_up)
    _check_modes(mixed_precision, interpret, x.dtype)
    guard = _GateUpSplits(blocks)
    if x.shape[1] != u_gate.shape[0]:
        raise ValueError("x/u_gate contraction dimensions do not match")
    layer = _cache.get("gu", (u_gate, v_gate, u_up, v_up), lambda: pack_svd_layer(u_gate, v_gate, u_up, v_up))
    with guard:
        return _finish(gate_up_packed(layer, x), x)


def xuv_matmul(x, u, v, *, mixed_precision=True, interpret=False):
    """[S, H] = (X.U).V (kernels/reference.py:75-82 fused_xuv_ref;
    pallas_ops.xuv_matmul, bench/profile_xuv.py:32-39)."""
    _validate_arrays(x, u, v)
    _check_modes(mixed_precision, interpret, x.dtype)
    if x.shape[1] != u.shape[0] or u.shape[1] != v.shape[0]:
        raise ValueError("x, U, V contraction dimensions do not match")
    layer = _cache.get("xuv", (u, v), lambda: pack_svd_layer(u_down=u, v_down=v))
    return _finish(xuv_packed(layer, x), x)


fused_xuv = xuv_matmul


def svd_mlp(x, u_gate, v_gate, u_up, v_up, u_down, v_down, *, gate_up_blocks=None, mixed_precision=True,
            interpret=False, residual=None):
    """Full SVD SwiGLU block (kernels/reference.py:85-93; pallas_ops.svd_mlp,
    bench/latency.py:402-404, models/modeling_llama.py:851-862)."""
    _validate_arrays(x, u_gate, v_gate, u_up, v_up, u_down, v_down)
    _check_modes(mixed_precision, interpret, x.dtype)
    guard = _GateUpSplits(gate_up_blocks)
    if x.shape[1] != u_gate.shape[0]:
        raise ValueError("x/u_gate contraction dimensions do not match")
    layer = _cache.get("svd", (u_gate, v_gate, u_up, v_up, u_down, v_down),
                       lambda: pack_svd_layer(u_gate, v_gate, u_up, v_up, u_down, v_down))
    with guard:
        return _finish(svd_mlp_packed(layer, x, residual=residual), x)


def contracted_svd_mlp(x, u_gate, v_gate, u_up, v_up, u_down, v_down, *, gate_up_blocks=None,
                       mixed_precision=True, interpret=False, residual=None):
    """pallas_ops.contracted_svd_mlp (models/modeling_llama.py:865-886,
    bench/all_mlp_layers.py:491-503): the layer with gate/up fused through
    . u_down (svdmlp_forward_contracted).  At decode sizes (<= 16 tokens) each
    SwiGLU tile of H stays in shared memory and is multiplied by its u_down
    slice in the same unit; above that the two-operator path runs, where H
    stays in the 126 MB L2 between the kernels."""
    _validate_arrays(x, u_gate, v_gate, u_up, v_up, u_down, v_down)
    _check_modes(mixed_precision, interpret, x.dtype)
    guard = _GateUpSplits(gate_up_blocks)
    if x.shape[1] != u_gate.shape[0]:
        raise ValueError("x/u_gate contraction dimensions do not match")
    layer = _cache.get("svd", (u_gate, v_gate, u_up, v_up, u_down, v_down),
                       lambda: pack_svd_layer(u_gate, v_gate, u_up, v_up, u_down, v_down))
    with guard:
        return _finish(contracted_mlp_packed(layer, x, residual=residual), x)


def dense_mlp(x, w_gate, w_up, w_down, *, mixed_precision=True, interpret=False, residual=None):
    """Dense SwiGLU from the same kernels (kernels/reference.py:96-106;
    pallas_ops.dense_mlp, models/modeling_llama.py:930-937)."""
    _validate_arrays(x, w_gate, w_up, w_down)
    _check_modes(mixed_precision, interpret, x.dtype)
    if x.shape[1] != w_gate.shape[0]:
        raise ValueError("x/w_gate contraction dimensions do not match")
    layer = _cache.get("dense", (w_gate, w_up, w_down), lambda: pack_dense_layer(w_gate, w_up, w_down))
    return _finish(dense_mlp_packed(layer, x, residual=residual), x)


def _pack_transposed(w: torch.Tensor) -> torch.Tensor:
    """w [K, N] -> w^T [N, K_pad] bf16 (K-major), K padded to 8 elements."""
    k, n = w.shape
    kp = (k + 7) // 8 * 8
    wt = torch.empty((n, kp), dtype=torch.bfloat16, device=w.device)
    wb = _bf16(w).contiguous()
    _lib.check(_lib.load().svdmlp_transpose_pack(wb.data_ptr(), _ld(wb), k, n, wt.data_ptr(), kp, n, kp,
                                                 _stream(w.device)), "transpose_pack")
    return wt


def dense_matmul(x, w, mixed_precision=True, interpret=False):
    """[M, N] = X[M, K] . W[K, N] on the tcgen05 GEMM (pallas_ops.dense_matmul,
    bench/diagnose_down.py:121; test_speedup.py:548-615)."""
    _validate_arrays(x, w)
    _check_modes(mixed_precision, interpret, x.dtype)
    if x.shape[1] != w.shape[0]:
        raise ValueError("x/w contraction dimensions do not match")
    m, k = x.shape
    n = w.shape[1]
    wt = _cache.get("gemm", (w,), lambda: _pack_transposed(w))
    xb = _bf16(x)
    if not (xb.stride(1) == 1 and xb.stride(0) % 8 == 0 and xb.data_ptr() % 16 == 0):
        kp = (k + 7) // 8 * 8
        xp = torch.zeros((m, kp), dtype=torch.bfloat16, device=x.device)
        xp[:, :k] = xb
        xb = xp
    n_pad = (n + 7) // 8 * 8
    c = torch.empty((m, n_pad), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    need = lib.svdmlp_gemm_workspace_bytes(m, n, k)
    ws = workspace_for(x.device, need)
    _lib.check(lib.svdmlp_gemm(xb.data_ptr(), xb.stride(0), wt.data_ptr(), wt.stride(0), c.data_ptr(), n_pad,
                               m, n, k, ws.ptr, ws.nbytes, _stream(x.device)), "dense_matmul")
    return _finish(c[:, :n], x)
