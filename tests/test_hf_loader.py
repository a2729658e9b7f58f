"""The safetensors checkpoint loader (models/hf_svd.py:13-196 of the reference):
key names, the [out, in] -> operand transpose with the v/u order reversed,
validation and errors, on a synthetic two-shard checkpoint written here."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import svdmlp_oracle as orc
from svdflash_b200.models import hf_svd

D, FF, R = 64, 96, 24


def _linear_weights(seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    mk = lambda o, i: (torch.randn(o, i, generator=g) / i ** 0.5).to(dtype)  # noqa: E731  [out, in]
    return {"gate_v_proj.weight": mk(R, D), "gate_u_proj.weight": mk(FF, R), "up_v_proj.weight": mk(R, D),
            "up_u_proj.weight": mk(FF, R), "down_v_proj.weight": mk(R, FF), "down_u_proj.weight": mk(D, R)}


def _write(tmp_path, layers=2, config_extra=None, drop_key=None, drop_shard=False, weights=None):
    from safetensors.torch import save_file
    config = {"hidden_size": D, "intermediate_size": FF, "num_hidden_layers": layers, "hidden_act": "silu"}
    config.update(config_extra or {})
    (tmp_path / "config.json").write_text(json.dumps(config))
    weight_map, per_layer = {}, []
    for layer in range(layers):
        w = weights[layer] if weights else _linear_weights(100 + layer)
        per_layer.append(w)
        shard = f"model-{layer + 1:05d}-of-{layers:05d}.safetensors"
        tensors = {f"model.layers.{layer}.mlp.{k}": v for k, v in w.items()}
        if drop_key and drop_key in tensors:
            del tensors[drop_key]
        if not (drop_shard and layer == layers - 1):
            save_file(tensors, str(tmp_path / shard))
        for k in tensors:
            weight_map[k] = shard
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    return per_layer


def test_factor_keys_and_metadata(tmp_path):
    assert hf_svd.factor_keys(3)[0] == "model.layers.3.mlp.gate_v_proj.weight"
    with pytest.raises(ValueError, match="non-negative"):
        hf_svd.factor_keys(-1)
    with pytest.raises(FileNotFoundError, match="missing checkpoint config"):
        hf_svd.checkpoint_metadata(tmp_path)
    _write(tmp_path)
    config, index = hf_svd.checkpoint_metadata(tmp_path)
    assert config["hidden_size"] == D and len(index["weight_map"]) == 12


def test_inspect_reads_headers_only(tmp_path):
    _write(tmp_path)
    info = hf_svd.inspect_mlp_checkpoint(tmp_path)
    assert info["selected_layers"] == [0, 1] and len(info["shards"]) == 2
    lay = info["layers"][1]
    assert lay["rank"] == R and lay["dtype"] == "BF16"
    assert lay["factor_bytes"] == 2 * (2 * D * R + 2 * R * FF + FF * R + R * D)
    assert lay["tensors"][0]["shape"] == [R, D]


def test_load_transposes_and_orders_factors(tmp_path):
    per_layer = _write(tmp_path)
    (f1,) = hf_svd.load_mlp_factors(tmp_path, [1], device="cpu")
    w = per_layer[1]
    want = [w["gate_v_proj.weight"].t(), w["gate_u_proj.weight"].t(), w["up_v_proj.weight"].t(),
            w["up_u_proj.weight"].t(), w["down_v_proj.weight"].t(), w["down_u_proj.weight"].t()]
    for got, ref in zip(f1, want):
        assert got.is_contiguous() and torch.equal(got, ref)
    assert [tuple(t.shape) for t in f1] == [(D, R), (R, FF), (D, R), (R, FF), (FF, R), (R, D)]


def test_loader_errors(tmp_path):
    _write(tmp_path, drop_key="model.layers.1.mlp.up_u_proj.weight")
    with pytest.raises(KeyError, match="missing MLP factors"):
        hf_svd.load_mlp_factors(tmp_path, [1], device="cpu")
    with pytest.raises(ValueError, match="at least one layer"):
        hf_svd.load_mlp_factors(tmp_path, [], device="cpu")
    with pytest.raises(ValueError, match=r"layer indices must be in \[0, 2\)"):
        hf_svd.inspect_mlp_checkpoint(tmp_path, [2])
    with pytest.raises(ValueError, match="without duplicates"):
        hf_svd.inspect_mlp_checkpoint(tmp_path, [0, 0])


def test_loader_rejects_missing_shards_bias_and_bad_factors(tmp_path):
    d1, d2, d3, d4 = (tmp_path / n for n in ("a", "b", "c", "d"))
    for p in (d1, d2, d3, d4):
        p.mkdir()
    _write(d1, drop_shard=True)
    with pytest.raises(FileNotFoundError, match="shards required"):
        hf_svd.load_mlp_factors(d1, [1], device="cpu")
    _write(d2, config_extra={"mlp_bias": True})
    with pytest.raises(ValueError, match="bias-free SwiGLU"):
        hf_svd.inspect_mlp_checkpoint(d2)
    bad = _linear_weights(7)
    bad["down_u_proj.weight"] = bad["down_u_proj.weight"][:, :R - 1].contiguous()  # wrong rank
    _write(d3, layers=1, weights=[bad])
    with pytest.raises(ValueError, match="invalid transposed MLP factor shapes"):
        hf_svd.load_mlp_factors(d3, [0], device="cpu")
    mixed = _linear_weights(8)
    mixed["up_u_proj.weight"] = mixed["up_u_proj.weight"].float()
    _write(d4, layers=1, weights=[mixed])
    with pytest.raises(TypeError, match="dtypes differ"):
        hf_svd.load_mlp_factors(d4, [0], device="cpu")


@pytest.mark.gpu
def test_loaded_layer_runs_on_gpu(tmp_path, cuda_device):
    """A loaded layer, packed, matches the oracle on the checkpoint's factors."""
    from helpers import assert_close, to_dev, to_np
    _write(tmp_path)
    mlps = hf_svd.load_svd_mlps(tmp_path, [0, 1], device=cuda_device)
    x = orc.bf16_round(np.random.default_rng(5).standard_normal((40, D), dtype=np.float32))
    factors = hf_svd.load_mlp_factors(tmp_path, [1], device="cpu")[0]
    y = mlps[1](to_dev(x, cuda_device))
    assert_close(to_np(y), orc.svd_mlp(x, *[f.float().numpy() for f in factors]), what="checkpoint layer 1")
