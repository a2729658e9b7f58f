"""The CPU oracle against the golden vectors produced by the reference's own
kernels/reference.py (tests/golden/make_golden.py)."""
from __future__ import annotations

import hashlib
import json
import pathlib

import numpy as np
import pytest

import svdmlp_oracle as orc

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
INDEX = json.loads((GOLDEN / "index.json").read_text())
CASES = [k for k in INDEX if k != "low_rank_dim"]
NAMES = ("x", "u_gate", "v_gate", "u_up", "v_up", "u_down", "v_down", "w_gate", "w_up", "w_down")


def _inputs(name):
    meta = INDEX[name]
    z = np.load(GOLDEN / f"{name}.npz")
    if meta["full"]:
        return {k: orc.from_bf16_bits(z[k]) for k in NAMES}, z
    x, f = orc.make_inputs(meta["seed"], meta["S"], meta["H"], meta["I"], meta["R"])
    wg, wu, wd = orc.make_dense(meta["seed"] + 1000, meta["H"], meta["I"])
    ins = dict(zip(NAMES, (x, *f, wg, wu, wd)))
    h = hashlib.sha256()
    for k in sorted(ins):
        h.update(k.encode())
        h.update(orc.bf16_bits(ins[k]).tobytes())
    assert h.hexdigest() == bytes(z["inputs_sha256"]).decode(), "seeded inputs no longer reproduce the fixture"
    return ins, z


def _check(got, z, key, full):
    if full:
        np.testing.assert_allclose(got, z[key], rtol=2e-5, atol=2e-5 * float(np.abs(z[key]).max()))
    else:
        np.testing.assert_allclose(got[:8], z[key + "_head"], rtol=2e-5, atol=2e-5 * float(np.abs(z[key + "_head"]).max()))
        assert abs(float(np.linalg.norm(got.astype(np.float64))) - float(z[key + "_norm"])) <= 1e-5 * float(z[key + "_norm"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_golden(name):
    ins, z = _inputs(name)
    full = INDEX[name]["full"]
    f = [ins[k] for k in ("u_gate", "v_gate", "u_up", "v_up", "u_down", "v_down")]
    gu = orc.fused_gate_up(ins["x"], *f[:4])
    _check(gu, z, "gate_up", full)
    _check(orc.fused_xuv(gu, f[4], f[5]), z, "xuv", full)
    _check(orc.svd_mlp(ins["x"], *f), z, "svd_mlp", full)
    _check(orc.dense_mlp(ins["x"], ins["w_gate"], ins["w_up"], ins["w_down"]), z, "dense_mlp", full)
    np.testing.assert_allclose(orc.silu(z["silu_in"]), z["silu_out"], rtol=1e-6, atol=1e-7)


def test_low_rank_dim_table():
    for key, want in INDEX["low_rank_dim"].items():
        h, i, c = key.split("_")
        assert orc.low_rank_dim(int(h), int(i), float(c)) == want


def test_benchmark_ranks():
    # r = floor(ratio * in * out / (in + out)) for the benchmark configurations
    assert [orc.benchmark_rank(4096, 14336, c) for c in (0.4, 0.6, 0.8, 0.9)] == [1274, 1911, 2548, 2867]
    assert orc.benchmark_rank(8192, 28672, 0.8) == 5097


def test_bf16_round_is_nearest_even():
    a = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 65504.0, 1e-30], dtype=np.float32)
    import torch
    want = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(orc.bf16_round(a), want)


def test_error_metrics_and_tolerance():
    ref = np.ones((4, 4), dtype=np.float32)
    m = orc.error_metrics(ref * (1 + 1e-3), ref)
    assert m["rel_fro"] == pytest.approx(1e-3, rel=1e-3)
    assert orc.within_tolerance(m)
    bad = ref.copy()
    bad[0, 0] = 1.1
    assert not orc.within_tolerance(orc.error_metrics(bad, ref))
    assert orc.error_metrics(np.full_like(ref, np.nan), ref)["nonfinite"] == 16


def test_planted_mistake_is_caught():
    """A wrong SiLU planted in the oracle's arithmetic fails the tolerance."""
    x, f = orc.make_inputs(3, 16, 64, 96, 40)
    good = orc.svd_mlp(x, *f)
    g = (x @ f[0]) @ f[1]
    u = (x @ f[2]) @ f[3]
    wrong = ((g * u) @ f[4]) @ f[5]            # SiLU dropped
    assert not orc.within_tolerance(orc.error_metrics(wrong, good))
