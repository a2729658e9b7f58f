"""GPU smoke of the B200 ports of the reference's benches (latency, tune):
their flags parse, every arm runs through the facade imports, and the report
keeps the reference's keys (bench/latency.py:112-126, 269-314, 536-558;
bench/tune.py:260-278)."""
from __future__ import annotations

import json

import pytest

pytestmark = pytest.mark.gpu

TIMING_KEYS = {"latency_ms_avg", "latency_ms_p50", "latency_ms_p90", "latency_ms_p95", "latency_ms_p99",
               "latency_ms_p100", "latency_ms_min", "iterations", "measured_seconds",
               "throughput_tokens_per_second"}


def test_latency_port_all_arms(cuda_device, tmp_path):
    from svdflash_b200.bench import latency
    out = tmp_path / "lat.json"
    rep = latency.main(["--models", "llama-3.2-3b", "--sequence-lengths", "1,300", "--benchmark", "all",
                        "--warmup", "1", "--iterations", "2", "--output", str(out)])
    assert json.loads(out.read_text())["benchmark_scope"] == "single_transformer_mlp_layer"
    names = {r["benchmark"] for r in rep["results"]}
    assert {"dense_mlp", "down_xuv", "fused_gate_up", "unfused_svd_mlp", "unfused_svd_mlp_b200",
            "two_kernel_svd_mlp", "contracted_hidden_svd_mlp", "vendor_gate_up", "vendor_down_xuv"} <= names
    for r in rep["results"]:
        assert TIMING_KEYS <= set(r) and r["latency_ms_avg"] > 0
        assert r["rank"] == 1792 and r["gate_up_blocks"]["bn"] in (128, 256)
    s = {(x["sequence_length"]): x for x in rep["speedups"]}
    assert {"speedup_vs_dense", "speedup_vs_unfused_svd", "speedup_contracted_vs_two_kernel"} <= set(s[300])


def test_tune_port_feeds_latency(cuda_device, tmp_path):
    from svdflash_b200.bench import latency, tune
    out = tmp_path / "tune.json"
    rep = tune.main(["--models", "llama-3.2-3b", "--sequence-lengths", "300", "--warmup", "1", "--iterations", "2",
                     "--output", str(out)])
    assert rep["best"] and all(r["status"] == "ok" for r in rep["records"]), rep["records"]
    assert {r["blocks"]["splits"] for r in rep["records"]} == {c["blocks"]["splits"] for c in rep["records"]}
    lat = latency.main(["--models", "llama-3.2-3b", "--sequence-lengths", "300", "--benchmark", "gate-up",
                        "--compress-ratio", "0.8", "--warmup", "1", "--iterations", "2",
                        "--tuning-config", str(out)])
    assert lat["tuned_workloads"] == 1
    assert lat["results"][-1]["gate_up_blocks"] == rep["best"][0]["blocks"]


def test_reference_api_numpy_in_numpy_out(cuda_device):
    """svdflash_tpu.kernels.reference on B200: the reference's golden operator
    names with NumPy arrays in and out (dtype of x kept), computed by the
    sm_100a kernels, within the north-star tolerance of the fp32 oracle."""
    import numpy as np

    import svdmlp_oracle as orc
    from helpers import assert_close, assert_close_bf16_output
    from svdflash_tpu.kernels import reference as ref_api
    x, f = orc.make_inputs(61, 40, 256, 512, 100)
    y = ref_api.svd_mlp_ref(x, *f)
    assert isinstance(y, np.ndarray) and y.dtype == np.float32 and y.shape == (40, 256)
    assert_close(y, orc.svd_mlp(x, *f), what="svd_mlp_ref")
    h = ref_api.fused_gate_up_ref(x, *f[:4])
    assert_close_bf16_output(h, orc.fused_gate_up(x, *f[:4]), what="fused_gate_up_ref")
    hb = orc.bf16_round(orc.fused_gate_up(x, *f[:4]))
    assert_close(ref_api.fused_xuv_ref(hb, f[4], f[5]), orc.fused_xuv(hb, f[4], f[5]), what="fused_xuv_ref")
    wg, wu, wd = orc.make_dense(62, 256, 512)
    assert_close(ref_api.dense_mlp_ref(x, wg, wu, wd), orc.dense_mlp(x, wg, wu, wd), what="dense_mlp_ref")
    np.testing.assert_allclose(ref_api.silu(np.linspace(-20, 20, 41, dtype=np.float32)),
                               orc.silu(np.linspace(-20, 20, 41, dtype=np.float32)), rtol=1e-6, atol=1e-6)
    assert ref_api.low_rank_dim(4096, 14336, 0.8) == orc.low_rank_dim(4096, 14336, 0.8)
