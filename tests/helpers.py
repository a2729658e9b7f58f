"""Shared helpers for the parity tests (host side only)."""
from __future__ import annotations

import numpy as np
import torch

import svdmlp_oracle as orc


def to_dev(a: np.ndarray, device, dtype=torch.bfloat16) -> torch.Tensor:
    """fp32 array on the bf16 grid -> device tensor (exact)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device=device, dtype=dtype)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def assert_close(got, ref, rel=5e-3, max_abs_rms=2e-2, what=""):
    m = orc.error_metrics(got, ref)
    assert m["nonfinite"] == 0, f"{what}: non-finite outputs {m}"
    assert m["rel_fro"] <= rel, f"{what}: rel-Frobenius {m['rel_fro']:.3e} > {rel} ({m})"
    assert m["max_abs_over_rms"] <= max_abs_rms, f"{what}: max-abs/RMS {m['max_abs_over_rms']:.3e} > {max_abs_rms} ({m})"
    return m


def assert_close_bf16_output(got, ref, rel=5e-3, max_abs_rms=2e-2, what=""):
    """Tolerance for an operator whose own output is a bf16 intermediate
    (the standalone gate/up H): |got - ref| <= 2e-2 * RMS(ref) + 2^-7 * |ref|
    elementwise, i.e. the layer criterion plus one bf16 ulp of the reference
    value, because H is heavy-tailed and a single bf16 rounding of its largest
    entries (which the reference's fused_gate_up_ref also applies with
    .astype(x.dtype)) already exceeds 2e-2 * RMS."""
    m = orc.error_metrics(got, ref)
    assert m["nonfinite"] == 0, f"{what}: non-finite outputs {m}"
    assert m["rel_fro"] <= rel, f"{what}: rel-Frobenius {m['rel_fro']:.3e} > {rel} ({m})"
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    bound = max_abs_rms * m["rms"] + 2.0 ** -7 * np.abs(r)
    worst = float(np.max(np.abs(g - r) - bound))
    assert worst <= 0, f"{what}: elementwise bound exceeded by {worst:.3e} ({m})"
    return m
