"""The C-ABI library loads and exports every symbol include/svdmlp.h
declares; host-side argument checks return the documented status codes.
No compute call reaches a GPU here."""
from __future__ import annotations

import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "svdmlp.h"


@pytest.fixture(scope="module")
def lib():
    from svdflash_b200 import _build, _lib
    if _build.is_stale():
        _build.build()
    return _lib.load()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(svdmlp_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_matches_header(lib):
    from svdflash_b200 import _lib
    assert set(_lib.SIGNATURES) == set(declared_functions())


def test_layout_sizes(lib):
    from svdflash_b200 import _lib
    L = _lib.Layout()
    assert lib.svdmlp_layout_init(ctypes.byref(L), 4096, 14336, 2867, 2867) == 0
    assert (L.rp_gu, L.rp_d, L.ld_d, L.ld_ff, L.ud_f16) == (2880, 2872, 4096, 14336, 1)

    def tiled(n, k):  # 16-row x 64-column tiles, 2 bytes per element
        return -(-n // 16) * 16 * (-(-k // 64) * 64) * 2
    # w1 [2*rp_gu, d] + vg, vu [ff, r] + ud [r, ff] + vd [d, r]
    expect = tiled(2 * 2880, 4096) + 2 * tiled(14336, 2867) + tiled(2867, 14336) + tiled(4096, 2867)
    # plus the 256-byte pack status block, each matrix rounded up to 256 bytes
    assert L.packed_bytes == pytest.approx(expect + 256, abs=5 * 256)
    for off in (L.off_w1, L.off_vg, L.off_vu, L.off_ud, L.off_vd, L.off_status):
        assert off % 256 == 0
    assert L.off_status + 256 == L.packed_bytes
    assert lib.svdmlp_workspace_bytes(ctypes.byref(L), 1024) > 0
    D = _lib.Layout()
    assert lib.svdmlp_dense_layout_init(ctypes.byref(D), 129, 137) == 0
    assert (D.ld_d, D.ld_ff, D.kind) == (136, 144, _lib.KIND_DENSE)
    X = _lib.Layout()
    assert lib.svdmlp_layout_init(ctypes.byref(X), 513, 1025, 0, 513) == 0
    assert X.ud_f16 == 0 and X.r_gu == 0


@pytest.mark.parametrize("args", [(0, 10, 4, 4), (10, -1, 4, 4), (10, 10, -1, 4), (10, 10, 0, 0)])
def test_layout_rejects_bad_sizes(lib, args):
    from svdflash_b200 import _lib
    L = _lib.Layout()
    assert lib.svdmlp_layout_init(ctypes.byref(L), *args) == _lib.ERR_INVALID_VALUE


def test_entry_points_reject_bad_arguments(lib):
    from svdflash_b200 import _lib
    L = _lib.Layout()
    assert lib.svdmlp_layout_init(ctypes.byref(L), 64, 96, 40, 40) == 0
    # null pointers / non-positive M fail before any device work
    assert lib.svdmlp_forward(ctypes.byref(L), None, None, 64, 8, None, 64, None, 0, None, 0, None) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_gate_up(ctypes.byref(L), 1, 1, 64, 0, 1, 96, 1, 1 << 20, None) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_xuv(ctypes.byref(L), 1, 1, 10, 4, 1, 64, 1, 1 << 20, None) == _lib.ERR_INVALID_VALUE  # ld_h < ff
    assert lib.svdmlp_workspace_init(None, 0, None) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_gemm(None, 8, None, 8, None, 8, 4, 4, 4, None, 0, None) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_set_split_override(9, 1) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_set_layer_decode(65) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_set_decode_overlap(9) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_set_pair_min_m(130) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_set_decode_prefetch(-1, 0) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_set_prefill_chain(-1) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_set_decode_contract(17) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_set_split_tail(2) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_rmsnorm(None, 8, None, None, 8, 1, 8, 1e-5, None) == _lib.ERR_INVALID_VALUE
    # misaligned output of the fp32 partial
    assert lib.svdmlp_forward_partial(ctypes.byref(L), 1, 1, 64, 4, 2, 40, 256, 1 << 20, None) == _lib.ERR_ALIGNMENT
    # peer memory: checked before any CUDA call
    sig = lib.svdmlp_peer_signal_bytes()
    assert sig >= 16 * 1024 and sig % 256 == 0
    ptr, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
    assert lib.svdmlp_peer_alloc(sig, ctypes.byref(ptr), handle) == _lib.ERR_INVALID_VALUE  # no data area
    assert lib.svdmlp_peer_open(None, ctypes.byref(ptr)) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_peer_close(None) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_peer_free(None) == _lib.ERR_INVALID_VALUE
    bases = (ctypes.c_void_p * 2)(4096, 8192)
    assert lib.svdmlp_peer_allreduce_f16(None, 2, 0, sig, 8, 8, 8, sig, None) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_peer_allreduce_f16(bases, 9, 0, sig, 8, 8, 8, sig, None) == _lib.ERR_INVALID_VALUE   # world > 8
    assert lib.svdmlp_peer_allreduce_f16(bases, 2, 2, sig, 8, 8, 8, sig, None) == _lib.ERR_INVALID_VALUE   # rank >= world
    assert lib.svdmlp_peer_allreduce_f16(bases, 2, 0, 0, 8, 8, 8, sig, None) == _lib.ERR_INVALID_VALUE     # in the signal area
    assert lib.svdmlp_peer_allreduce_f16(bases, 2, 0, sig, 8, 12, 16, sig, None) == _lib.ERR_INVALID_VALUE  # c % 8
    odd = (ctypes.c_void_p * 2)(4096, 8200)
    assert lib.svdmlp_peer_allgather(odd, 2, 0, sig, 8, 16, 16, None) == _lib.ERR_ALIGNMENT
    assert lib.svdmlp_peer_allgather(bases, 2, 0, sig, 8, 24, 32, None) == _lib.ERR_INVALID_VALUE     # 16-byte rows
    assert lib.svdmlp_peer_reduce_scatter_f16(bases, 2, 0, sig, 8, 8, 8, sig, None, 8, None) == _lib.ERR_INVALID_VALUE
    assert lib.svdmlp_peer_allreduce_f16(bases, 2, 0, sig, 8, 8, 8, 8, None) == _lib.ERR_INVALID_VALUE  # scratch
    assert lib.svdmlp_peer_scratch_bytes(2, 37, 24) == 2 * 2 * 19 * 24 * 2
    assert lib.svdmlp_peer_check_status(None, None) == _lib.ERR_INVALID_VALUE
    # the fused exchange: slot geometry and offsets checked before any CUDA call
    assert lib.svdmlp_peer_slots_bytes(2, 256, 2872) == 2 * 2 * 256 * 2872 * 2
    assert lib.svdmlp_peer_slots_bytes(2, 256, 2870) == 0 and lib.svdmlp_peer_slots_bytes(9, 256, 8) == 0
    assert lib.svdmlp_forward_partial_f16_peer(ctypes.byref(L), 1, 1, 64, 8, bases, 2, 0, sig, 4, 40, None, 0,
                                               None) == _lib.ERR_INVALID_VALUE  # M > slot_rows
    assert lib.svdmlp_forward_partial_f16_peer(ctypes.byref(L), 1, 1, 64, 4, bases, 2, 0, sig, 4, 36, None, 0,
                                               None) == _lib.ERR_INVALID_VALUE  # ld_slot < r_d
    assert lib.svdmlp_forward_partial_f16_peer(ctypes.byref(L), 1, 1, 64, 4, bases, 2, 0, 0, 4, 40, None, 0,
                                               None) == _lib.ERR_INVALID_VALUE  # slots in the signal area
    assert lib.svdmlp_peer_sum_f16(bases, 2, 0, sig, 4, 8, 8, 8, ctypes.c_void_p(4096), 8, None) == \
        _lib.ERR_INVALID_VALUE  # m > slot_rows
    assert lib.svdmlp_peer_sum_f16(bases, 2, 0, sig, 8, 8, 12, 16, ctypes.c_void_p(4096), 16, None) == \
        _lib.ERR_INVALID_VALUE  # c % 8
    assert lib.svdmlp_peer_sum_f16(bases, 2, 0, sig, 8, 8, 8, 8, ctypes.c_void_p(4100), 8, None) == \
        _lib.ERR_ALIGNMENT


def test_status_strings(lib):
    from svdflash_b200 import _lib
    for code in range(0, -11, -1):
        assert lib.svdmlp_status_string(code) != b"unknown status"
    assert b"fp16 range" in lib.svdmlp_status_string(_lib.ERR_RANGE)
    assert b"positive" in lib.svdmlp_status_string(_lib.ERR_INVALID_VALUE)
    assert b"SMEM/TMEM budget" in lib.svdmlp_status_string(_lib.ERR_BUDGET)


def test_plan_info_is_deterministic(lib):
    out = (ctypes.c_int * 6)()
    assert lib.svdmlp_plan_info(1, 1024, 14336, 2867, out) == 0
    assert list(out)[:3] == [4, 56, 45]           # 256-row CTA-pair tiles, 256 per branch, 64-wide k-blocks
    assert out[3] == 1
    assert lib.svdmlp_plan_info(1, 1, 14336, 2867, out) == 0
    assert out[0] == 1 and out[3] >= 1 and out[4] == out[1] * out[3]


def test_decode_plans_split_one_branch_stages_per_sm(lib):
    """Per-stage decode plans above 16 tokens: one-branch stages split to at
    least 1.2 units per SM (148 SMs without a GPU), the dual gate/up stage
    stays unsplit; the 8B layer at ratio 0.9 gives the measured best splits
    X.[u_g,u_u] 4, H.u_down 8."""
    out = (ctypes.c_int * 6)()
    for m in (32, 128):
        assert lib.svdmlp_plan_info(0, m, 5760, 4096, out) == 0      # X.[u_g|u_u]: 45 tiles
        assert out[1] == 45 and out[3] == 4
        assert lib.svdmlp_plan_info(2, m, 2867, 14336, out) == 0     # H.u_down: 23 tiles
        assert out[1] == 23 and out[3] == 8 and out[1] * out[3] >= 1.2 * 148
        assert lib.svdmlp_plan_info(1, m, 14336, 2867, out) == 0     # dual gate/up
        assert out[3] == 1


def test_status_mapping_to_exceptions():
    from svdflash_b200 import _lib
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_SHAPE_MISMATCH)
    with pytest.raises(TypeError):
        _lib.check(_lib.ERR_DTYPE)
    with pytest.raises(_lib.SvdMlpError):
        _lib.check(_lib.ERR_DEVICE_TIMEOUT)
    with pytest.raises(_lib.SvdMlpRangeError):
        _lib.check(_lib.ERR_RANGE)
    with pytest.raises(FloatingPointError):
        _lib.check(_lib.ERR_RANGE)
    _lib.check(_lib.OK)
