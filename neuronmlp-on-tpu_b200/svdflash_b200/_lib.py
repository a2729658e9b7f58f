"""ctypes binding of the C ABI in ``include/svdmlp.h`` (``libsvdmlp.so``).

This is the only path to the kernels: there is no CPU or PyTorch fallback.
If the shared library is missing the import fails loudly.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_void_p

from . import _build

OK = 0
ERR_INVALID_VALUE = -1
ERR_SHAPE_MISMATCH = -2
ERR_ALIGNMENT = -3
ERR_DTYPE = -4
ERR_WORKSPACE = -5
ERR_DEVICE_TIMEOUT = -6
ERR_CUDA = -7
ERR_BUDGET = -8
ERR_DEVICE = -9
ERR_RANGE = -10

KIND_SVD = 1
KIND_DENSE = 2

# Stage ids of svdmlp_set_split_override / svdmlp_plan_info.
STAGE_XU, STAGE_GATE_UP, STAGE_DOWN_U, STAGE_DOWN_V, STAGE_DENSE_GU, STAGE_DENSE_DOWN, STAGE_GEMM = range(7)


class Layout(ctypes.Structure):
    """Mirror of ``svdmlp_layout``."""

    _fields_ = [
        ("kind", c_int32),
        ("d", c_int32),
        ("ff", c_int32),
        ("r_gu", c_int32),
        ("r_d", c_int32),
        ("rp_gu", c_int32),
        ("rp_d", c_int32),
        ("ld_d", c_int32),
        ("ld_ff", c_int32),
        ("ud_f16", c_int32),
        ("off_w1", c_int64),
        ("off_vg", c_int64),
        ("off_vu", c_int64),
        ("off_ud", c_int64),
        ("off_vd", c_int64),
        ("off_status", c_int64),
        ("packed_bytes", c_int64),
    ]


LP = POINTER(Layout)
V = c_void_p
I64 = c_int64

# name -> (restype, argtypes); the exact set declared in include/svdmlp.h.
SIGNATURES = {
    "svdmlp_status_string": (c_char_p, [c_int]),
    "svdmlp_last_cuda_error": (c_int, []),
    "svdmlp_layout_init": (c_int, [LP, c_int, c_int, c_int, c_int]),
    "svdmlp_dense_layout_init": (c_int, [LP, c_int, c_int]),
    "svdmlp_pack": (c_int, [LP, V, I64, V, I64, V, I64, V, I64, V, I64, V, I64, V, V]),
    "svdmlp_dense_pack": (c_int, [LP, V, I64, V, I64, V, I64, V, V]),
    "svdmlp_workspace_bytes": (c_int64, [LP, c_int]),
    "svdmlp_workspace_init": (c_int, [V, I64, V]),
    "svdmlp_check_device_status": (c_int, [V, I64, V]),
    "svdmlp_pack_status": (c_int, [LP, V, V]),
    "svdmlp_gate_up": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V]),
    "svdmlp_xuv": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V]),
    "svdmlp_forward": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V, I64, V]),
    "svdmlp_dense_forward": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V, I64, V]),
    "svdmlp_forward_contracted": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V, I64, V]),
    "svdmlp_forward_block": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V, c_float, V, I64, V]),
    "svdmlp_row_sumsq": (c_int, [V, I64, c_int, c_int, V, I64, V]),
    "svdmlp_pack_block": (c_int, [LP, V, V, I64, V, I64, V, I64, V, I64, V, I64, V, I64, V, V]),
    "svdmlp_set_decode_contract": (c_int, [c_int]),
    "svdmlp_down_partial": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V]),
    "svdmlp_forward_partial": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V]),
    "svdmlp_down_finish": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V, I64, V]),
    "svdmlp_forward_partial_f16": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V]),
    "svdmlp_down_finish_f16": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V, I64, V]),
    "svdmlp_xu_project": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V]),
    "svdmlp_partial_from_xu_f16": (c_int, [LP, V, V, I64, c_int, V, I64, V, I64, V]),
    "svdmlp_xuv_noalloc": (c_int, [LP, V, V, I64, c_int, V, I64, V]),
    "svdmlp_xuv_noalloc_status": (c_int, [V]),
    "svdmlp_gemm": (c_int, [V, I64, V, I64, V, I64, c_int, c_int, c_int, V, I64, V]),
    "svdmlp_gemm_workspace_bytes": (c_int64, [c_int, c_int, c_int]),
    "svdmlp_transpose_pack": (c_int, [V, I64, c_int, c_int, V, I64, c_int, c_int, V]),
    "svdmlp_rmsnorm": (c_int, [V, I64, V, V, I64, c_int, c_int, c_float, V]),
    "svdmlp_debug_wait_timeout": (c_int, [V, I64, I64, V]),
    "svdmlp_set_split_override": (c_int, [c_int, c_int]),
    "svdmlp_set_split_tail": (c_int, [c_int]),
    "svdmlp_set_layer_decode": (c_int, [c_int]),
    "svdmlp_set_decode_overlap": (c_int, [c_int]),
    "svdmlp_set_pair_min_m": (c_int, [c_int]),
    "svdmlp_set_decode_prefetch": (c_int, [c_int, c_int]),
    "svdmlp_set_prefill_chain": (c_int, [c_int]),
    "svdmlp_set_trace_buffer": (c_int, [V, I64]),
    "svdmlp_plan_info": (c_int, [c_int, c_int, c_int, c_int, POINTER(c_int)]),
    "svdmlp_tile_info": (c_int, [c_int, c_int, POINTER(c_int)]),
    "svdmlp_stage_timing": (c_int, [c_int]),
    "svdmlp_stage_times": (c_int, [POINTER(ctypes.c_double), POINTER(c_int64), c_int]),
    "svdmlp_launch_count": (c_int64, []),
    "svdmlp_peer_signal_bytes": (c_int64, []),
    "svdmlp_peer_alloc": (c_int, [c_int64, POINTER(c_void_p), c_void_p]),
    "svdmlp_peer_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "svdmlp_peer_close": (c_int, [c_void_p]),
    "svdmlp_peer_free": (c_int, [c_void_p]),
    "svdmlp_peer_scratch_bytes": (c_int64, [c_int, c_int, c_int]),
    "svdmlp_peer_allreduce_f16": (c_int, [POINTER(c_void_p), c_int, c_int, c_int64, c_int, c_int, c_int64, c_int64,
                                          c_void_p]),
    "svdmlp_peer_reduce_scatter_f16": (c_int, [POINTER(c_void_p), c_int, c_int, c_int64, c_int, c_int, c_int64,
                                               c_int64, c_void_p, c_int64, c_void_p]),
    "svdmlp_peer_allgather": (c_int, [POINTER(c_void_p), c_int, c_int, c_int64, c_int, c_int64, c_int64, c_void_p]),
    "svdmlp_peer_check_status": (c_int, [c_void_p, c_void_p]),
    "svdmlp_peer_slots_bytes": (c_int64, [c_int, c_int, c_int64]),
    "svdmlp_forward_partial_f16_peer": (c_int, [LP, V, V, I64, c_int, POINTER(c_void_p), c_int, c_int, c_int64,
                                                c_int, c_int64, V, I64, V]),
    "svdmlp_peer_sum_f16": (c_int, [POINTER(c_void_p), c_int, c_int, c_int64, c_int, c_int, c_int, c_int64,
                                    c_void_p, c_int64, c_void_p]),
}

_lock = threading.Lock()
_lib = None


def lib_path():
    """The shared library to load: $SVDMLP_LIBRARY (another build of the same
    sources, e.g. a tile sweep) or the in-tree build."""
    import os
    import pathlib
    env = os.environ.get("SVDMLP_LIBRARY")
    return pathlib.Path(env) if env else _build.LIB_PATH


def load() -> ctypes.CDLL:
    """Loads libsvdmlp.so (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not path.exists():
                raise RuntimeError(
                    f"libsvdmlp.so not found at {path}; build it with __graft_entry__.build() "
                    "or python -m svdflash_b200._build (there is no CPU fallback)")
            lib = ctypes.CDLL(str(path))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class SvdMlpError(RuntimeError):
    """A device-side or CUDA failure reported by the library."""


class SvdMlpRangeError(SvdMlpError, FloatingPointError):
    """An fp16 intermediate (or an fp16-packed weight) exceeded 65504 or was
    NaN and was saturated: the result of that call is not trustworthy."""


def check(status: int, what: str = "") -> None:
    """Maps a C-ABI status to the exception types the reference raises."""
    if status == OK:
        return
    lib = load()
    msg = lib.svdmlp_status_string(status).decode()
    if what:
        msg = f"{what}: {msg}"
    if status == ERR_CUDA:
        msg += f" (cudaError {lib.svdmlp_last_cuda_error()})"
    if status in (ERR_INVALID_VALUE, ERR_SHAPE_MISMATCH, ERR_ALIGNMENT, ERR_WORKSPACE, ERR_BUDGET):
        raise ValueError(msg)
    if status == ERR_DTYPE:
        raise TypeError(msg)
    if status == ERR_RANGE:
        raise SvdMlpRangeError(msg)
    raise SvdMlpError(msg)
