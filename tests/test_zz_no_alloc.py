"""GPU test of svdmlp_xuv_noalloc, the XUV down operator that allocates
nothing (for callers that cannot allocate device memory, such as plugins whose
host runtime owns every device allocation).  It is called through the C ABI
and checked against the workspace-taking svdmlp_xuv, on two calls in a row,
within the parity tolerance of the other tests.  This file is collected last
so that a failure here cannot hide the results of the other tests."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import svdmlp_oracle as orc
from helpers import assert_close, assert_close_bf16_output, to_dev, to_np

pytestmark = pytest.mark.gpu


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _run_existing(lib, layer, h, dev):
    from svdflash_b200 import _lib
    m = h.shape[0]
    y = torch.empty(m, layer.d, dtype=torch.bfloat16, device=dev)
    ws = layer.workspace(m)
    _lib.check(lib.svdmlp_xuv(ctypes.byref(layer.layout), layer.packed.data_ptr(), h.data_ptr(), h.stride(0), m,
                              y.data_ptr(), y.stride(0), ws.ptr, ws.nbytes, _stream(dev)))
    return y


def _run_noalloc(lib, layer, h, dev):
    from svdflash_b200 import _lib
    m = h.shape[0]
    y = torch.full((m, layer.d), float("nan"), dtype=torch.bfloat16, device=dev)
    _lib.check(lib.svdmlp_xuv_noalloc(ctypes.byref(layer.layout), layer.packed.data_ptr(), h.data_ptr(),
                                      h.stride(0), m, y.data_ptr(), y.stride(0), _stream(dev)))
    return y


@pytest.mark.parametrize("kind,m,d,ff,r", [
    ("down_only", 64, 512, 1024, 300),     # bf16 u_down, no H conversion
    ("full_layer", 40, 256, 512, 120),     # fp16 u_down: H converted into the static scratch
    ("decode_8b", 128, 4096, 14336, 2867),  # split-K partials do not fit: unsplit GEMMs
    ("prefill", 384, 1024, 2048, 520),     # CTA-pair kernels
])
def test_noalloc_matches_workspace_entry_point(cuda_device, kind, m, d, ff, r):
    from svdflash_b200 import _lib
    from svdflash_b200.kernels import ops
    lib = _lib.load()
    x, f = orc.make_inputs(70 + m, m, d, ff, r)
    fd = [to_dev(a, cuda_device) for a in f]
    layer = ops.pack_svd_layer(u_down=fd[4], v_down=fd[5]) if kind == "down_only" else ops.pack_svd_layer(*fd)
    hb = orc.bf16_round(orc.fused_gate_up(x, *f[:4]))
    h = to_dev(hb, cuda_device)
    want = _run_existing(lib, layer, h, cuda_device)
    outs = [_run_noalloc(lib, layer, h, cuda_device) for _ in range(2)]   # two calls in a row
    torch.cuda.synchronize()
    ref = to_np(want)
    for i, y in enumerate(outs):
        # Both are bf16 roundings of fp32 sums; when the no-alloc call runs a
        # GEMM unsplit where the workspace call split K, the sums round in a
        # different order and may differ by one bf16 ulp, which the bf16-output
        # tolerance of the other tests allows.
        assert_close_bf16_output(to_np(y), ref, what=f"{kind} call {i}")
    assert_close(to_np(outs[0]), orc.fused_xuv(hb, f[4], f[5]), what=f"{kind} vs oracle")


def test_noalloc_rejects_sizes_beyond_the_static_scratch(cuda_device):
    from svdflash_b200 import _lib
    from svdflash_b200.kernels import ops
    lib = _lib.load()
    _, f = orc.make_inputs(80, 1, 512, 1024, 300)
    fd = [to_dev(a, cuda_device) for a in f]
    layer = ops.pack_svd_layer(u_down=fd[4], v_down=fd[5])
    m = 16384   # 2 * 16384 * 304 bytes of rank-r intermediate alone exceed 8 MiB
    h = torch.zeros(m, 1024, dtype=torch.bfloat16, device=cuda_device)
    y = torch.zeros(m, 512, dtype=torch.bfloat16, device=cuda_device)
    st = lib.svdmlp_xuv_noalloc(ctypes.byref(layer.layout), layer.packed.data_ptr(), h.data_ptr(), h.stride(0), m,
                                y.data_ptr(), y.stride(0), _stream(cuda_device))
    assert st == _lib.ERR_WORKSPACE
    assert b"workspace" in lib.svdmlp_status_string(st)


def test_noalloc_status_reports_and_clears(cuda_device):
    """svdmlp_xuv_noalloc_status reads the error block inside the library's
    static array (the caller has no workspace to pass): OK after a clean
    call, SVDMLP_ERR_RANGE after a call whose H holds a value fp16 cannot
    hold (the full-layer layout converts H to fp16), OK again once read."""
    from svdflash_b200 import _lib
    from svdflash_b200.kernels import ops
    lib = _lib.load()
    m, d, ff, r = 40, 256, 512, 120
    x, f = orc.make_inputs(95, m, d, ff, r)
    layer = ops.pack_svd_layer(*[to_dev(a, cuda_device) for a in f])
    hb = orc.bf16_round(orc.fused_gate_up(x, *f[:4]))
    y = _run_noalloc(lib, layer, to_dev(hb, cuda_device), cuda_device)
    assert lib.svdmlp_xuv_noalloc_status(_stream(cuda_device)) == _lib.OK
    assert_close(to_np(y), orc.fused_xuv(hb, f[4], f[5]), what="clean call")
    bad = hb.copy()
    bad[7, 11] = 3.0e5
    _run_noalloc(lib, layer, to_dev(bad, cuda_device), cuda_device)
    assert lib.svdmlp_xuv_noalloc_status(_stream(cuda_device)) == _lib.ERR_RANGE
    assert lib.svdmlp_xuv_noalloc_status(_stream(cuda_device)) == _lib.OK
