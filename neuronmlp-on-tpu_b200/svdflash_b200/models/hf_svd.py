"""SVD MLP factors from a sharded Hugging Face safetensors checkpoint.

Mirrors the reference's loader (models/hf_svd.py:13-196): the same function
names, key names, validation and errors, returning torch tensors (on the
device asked for) instead of JAX arrays.

A checkpoint stores each factor as a torch.nn.Linear weight, [out, in].  The
first projection of a pair is named ``*_v_proj`` and the second ``*_u_proj``;
the operators take natural matmul operands, so every tensor is transposed
and the v/u order is reversed: (gate_v^T, gate_u^T, up_v^T, up_u^T, down_v^T,
down_u^T) = (u_gate [d, r], v_gate [r, ff], u_up [d, r], v_up [r, ff],
u_down [ff, r], v_down [r, d]).
"""
from __future__ import annotations

import json
from contextlib import ExitStack
from pathlib import Path
from typing import Optional, Sequence

import torch

FACTOR_SUFFIXES = (
    "gate_v_proj.weight",
    "gate_u_proj.weight",
    "up_v_proj.weight",
    "up_u_proj.weight",
    "down_v_proj.weight",
    "down_u_proj.weight",
)

_DTYPES = {"BF16": torch.bfloat16, "F32": torch.float32}

__all__ = ["FACTOR_SUFFIXES", "checkpoint_metadata", "factor_keys", "validate_factor_shapes",
           "inspect_mlp_checkpoint", "load_mlp_factors", "load_svd_mlps"]


def _read_json(path: Path, what: str) -> dict:
    if not path.is_file():
        raise FileNotFoundError(f"missing {what}: {path}")
    return json.loads(path.read_text(encoding="utf-8"))


def checkpoint_metadata(model_path: str | Path) -> tuple[dict, dict]:
    """(config.json, model.safetensors.index.json) of a checkpoint directory;
    the index must carry a weight_map (the reference's checks and errors,
    models/hf_svd.py:23-37)."""
    root = Path(model_path)
    config = _read_json(root / "config.json", "checkpoint config")
    index_path = root / "model.safetensors.index.json"
    index = _read_json(index_path, "safetensors index")
    if "weight_map" in index:
        return config, index
    raise ValueError(f"safetensors index has no weight_map: {index_path}")


def factor_keys(layer_index: int) -> tuple[str, ...]:
    if layer_index < 0:
        raise ValueError(f"layer index must be non-negative, got {layer_index}")
    prefix = f"model.layers.{layer_index}.mlp."
    return tuple(prefix + suffix for suffix in FACTOR_SUFFIXES)


def _check_mlp_config(config: dict) -> None:
    if config.get("hidden_act", "silu") != "silu" or config.get("mlp_bias", False):
        raise ValueError("the fused kernel requires bias-free SwiGLU MLPs")


def validate_factor_shapes(factors: Sequence, *, hidden_size: int, intermediate_size: int) -> int:
    """Checks that six transposed factors chain as [d, r] [r, ff] [d, r]
    [r, ff] [ff, r] [r, d] with one dtype, and returns r (the reference's
    checks and errors, models/hf_svd.py:47-74)."""
    if len(factors) != 6:
        raise ValueError(f"expected six MLP factors, got {len(factors)}")
    shapes = [tuple(int(n) for n in f.shape) for f in factors]
    r = shapes[0][1]
    d, ff = hidden_size, intermediate_size
    # (rows, cols) of each factor in operator order: a pair chains in -> r -> out
    want = [(d, r), (r, ff)] * 2 + [(ff, r), (r, d)]
    if shapes != want:
        raise ValueError(f"invalid transposed MLP factor shapes; expected {tuple(want)}, got {tuple(shapes)}")
    kinds = sorted({str(f.dtype) for f in factors})
    if len(kinds) > 1:
        raise TypeError(f"MLP factor dtypes differ: {kinds}")
    return r


def _selected(config: dict, layer_indices: Optional[Sequence[int]]) -> tuple[int, ...]:
    num_layers = int(config["num_hidden_layers"])
    selected = tuple(range(num_layers)) if layer_indices is None else tuple(layer_indices)
    if not selected or len(set(selected)) != len(selected):
        raise ValueError("select at least one layer, without duplicates")
    if min(selected) < 0 or max(selected) >= num_layers:
        raise ValueError(f"layer indices must be in [0, {num_layers})")
    return selected


def _shard_names(model_path: Path, weight_map: dict, keys: Sequence[str]) -> list[str]:
    missing = [key for key in keys if key not in weight_map]
    if missing:
        raise KeyError(f"checkpoint is missing MLP factors: {missing}")
    names = sorted({weight_map[key] for key in keys})
    absent = [name for name in names if not (model_path / name).is_file()]
    if absent:
        raise FileNotFoundError("checkpoint shards required by the selected layers are missing: " + ", ".join(absent))
    return names


def inspect_mlp_checkpoint(model_path: str | Path, layer_indices: Optional[Sequence[int]] = None) -> dict:
    """Validates the shard headers of the selected layers without loading payloads."""
    from safetensors import safe_open

    model_path = Path(model_path)
    config, index = checkpoint_metadata(model_path)
    _check_mlp_config(config)
    hidden, intermediate = int(config["hidden_size"]), int(config["intermediate_size"])
    selected = _selected(config, layer_indices)
    weight_map = index["weight_map"]
    names = _shard_names(model_path, weight_map, [k for layer in selected for k in factor_keys(layer)])
    layers = []
    with ExitStack() as stack:
        shards = {name: stack.enter_context(safe_open(str(model_path / name), framework="pt")) for name in names}
        for layer in selected:
            descriptors, info = [], []
            for key in factor_keys(layer):
                view = shards[weight_map[key]].get_slice(key)
                shape, dtype = tuple(view.get_shape()), view.get_dtype()
                if len(shape) != 2 or dtype not in _DTYPES or min(shape) <= 0:
                    raise ValueError(f"unsupported MLP tensor {key}: {shape}, {dtype}")
                descriptors.append(torch.empty(shape[::-1], dtype=_DTYPES[dtype], device="meta"))
                info.append({"key": key, "shape": list(shape), "dtype": dtype, "shard": weight_map[key]})
            rank = validate_factor_shapes(descriptors, hidden_size=hidden, intermediate_size=intermediate)
            nbytes = sum(d.numel() * d.element_size() for d in descriptors)
            layers.append({"layer": layer, "rank": rank, "dtype": info[0]["dtype"], "factor_bytes": nbytes,
                           "tensors": info})
    return {"model_path": str(model_path.resolve()), "num_hidden_layers": int(config["num_hidden_layers"]),
            "hidden_size": hidden, "intermediate_size": intermediate, "selected_layers": list(selected),
            "shards": names, "layers": layers}


def load_mlp_factors(model_path: str | Path, layer_indices: Sequence[int],
                     device: str | torch.device = "cuda") -> tuple[tuple[torch.Tensor, ...], ...]:
    """Loads the selected layers' factors, transposed to the operator order
    (u_gate, v_gate, u_up, v_up, u_down, v_down), onto `device`."""
    try:
        from safetensors import safe_open
    except ImportError as error:  # pragma: no cover - installed in this image
        raise RuntimeError("loading real factors requires safetensors") from error

    model_path = Path(model_path)
    config, index = checkpoint_metadata(model_path)
    _check_mlp_config(config)
    weight_map = index["weight_map"]
    layer_indices = tuple(layer_indices)
    if not layer_indices:
        raise ValueError("at least one layer must be selected")
    names = _shard_names(model_path, weight_map, [k for layer in layer_indices for k in factor_keys(layer)])
    layers = []
    with ExitStack() as stack:
        shards = {name: stack.enter_context(safe_open(str(model_path / name), framework="pt")) for name in names}
        for layer in layer_indices:
            factors = tuple(shards[weight_map[key]].get_tensor(key).t().contiguous().to(device)
                            for key in factor_keys(layer))
            validate_factor_shapes(factors, hidden_size=int(config["hidden_size"]),
                                   intermediate_size=int(config["intermediate_size"]))
            layers.append(factors)
    return tuple(layers)


def load_svd_mlps(model_path: str | Path, layer_indices: Sequence[int], device: str | torch.device = "cuda"):
    """The selected layers as SvdLlamaMLP modules (factors packed once, the
    checkpoint tensors released)."""
    from .svd_mlp import SvdLlamaMLP

    return [SvdLlamaMLP(*factors) for factors in load_mlp_factors(model_path, layer_indices, device)]
