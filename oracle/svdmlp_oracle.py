"""CPU oracle for the SVD-compressed SwiGLU MLP -- TEST INFRASTRUCTURE ONLY.

A NumPy fp32 restatement of the reference's golden operators
(n-paradigm/NeuronMLP-on-TPU, kernels/reference.py).  It is the checker for
the B200 kernels: only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg may import it.  The product path (svdflash_b200 and
libsvdmlp.so) never calls it and has no CPU fallback.

Parity of this restatement is pinned against the reference itself:
tests/golden/make_golden.py imports kernels/reference.py, runs it on seeded
inputs, and stores the inputs and outputs under tests/golden/; the CPU test
suite checks this module against those fixtures.

Conventions follow the reference: u_* is the first factor [in, r], v_* the
second factor [r, out]; arrays are row-major; all math is fp32.
"""
from __future__ import annotations

import numpy as np


def low_rank_dim(hidden_size: int, intermediate_size: int, compress_ratio: float) -> int:
    """128-aligned rank (kernels/reference.py:21-34)."""
    numer = intermediate_size * hidden_size * compress_ratio
    denom = (intermediate_size + hidden_size) * 128
    return round(numer / denom) * 128


def benchmark_rank(in_features: int, out_features: int, ratio: float) -> int:
    """floor(ratio * in * out / (in + out)), the rank of the benchmark configs."""
    return int(ratio * in_features * out_features // (in_features + out_features))


def silu(x: np.ndarray) -> np.ndarray:
    """fp32 x * sigmoid(x) with the exponent argument kept <= 0 on both
    branches (kernels/reference.py:37-51)."""
    x32 = np.asarray(x, dtype=np.float32)
    e = np.exp(-np.abs(x32))                       # exp of a non-positive number
    sig = np.where(x32 >= 0, 1.0 / (1.0 + e), e / (1.0 + e))
    return (x32 * sig).astype(np.float32)


def _f32(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32)


def fused_gate_up(x, u_gate, v_gate, u_up, v_up) -> np.ndarray:
    """silu((x.u_gate).v_gate) * ((x.u_up).v_up) in fp32
    (kernels/reference.py:54-72; the output is left in fp32)."""
    x = _f32(x)
    gate = (x @ _f32(u_gate)) @ _f32(v_gate)
    up = (x @ _f32(u_up)) @ _f32(v_up)
    return silu(gate) * up


def fused_xuv(x, u, v) -> np.ndarray:
    """(x.u).v in fp32 (kernels/reference.py:75-82)."""
    return (_f32(x) @ _f32(u)) @ _f32(v)


def svd_mlp(x, u_gate, v_gate, u_up, v_up, u_down, v_down) -> np.ndarray:
    """Full layer: fused_xuv(fused_gate_up(x)) (kernels/reference.py:85-93)."""
    return fused_xuv(fused_gate_up(x, u_gate, v_gate, u_up, v_up), u_down, v_down)


def dense_mlp(x, w_gate, w_up, w_down) -> np.ndarray:
    """Dense SwiGLU (kernels/reference.py:96-106)."""
    x = _f32(x)
    return (silu(x @ _f32(w_gate)) * (x @ _f32(w_up))) @ _f32(w_down)


def rmsnorm(x, weight, eps: float = 1e-5) -> np.ndarray:
    """x * rsqrt(mean(x^2) + eps) * weight (the decoder norm,
    models/modeling_llama.py:245-262, and bench/e2e_block.py:72-75)."""
    x = _f32(x)
    rstd = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * rstd * _f32(weight)


def mlp_block(x, norm_w, factors, eps: float = 1e-5) -> np.ndarray:
    """x + svd_mlp(rmsnorm(x)): one block of the MLP-only stack."""
    return _f32(x) + svd_mlp(rmsnorm(x, norm_w, eps), *factors)


# ------------------------------------------------------- ff-sharded layer
def shard_factors(factors, rank: int, world: int):
    """ff-shard of (u_g, v_g, u_u, v_u, u_d, v_d): v_* column-sharded, u_down
    row-sharded, the rest replicated."""
    u_g, v_g, u_u, v_u, u_d, v_d = factors
    ff = v_g.shape[1]
    if ff % world:
        raise ValueError("ff must divide evenly across ranks")
    lo, hi = rank * ff // world, (rank + 1) * ff // world
    return u_g, v_g[:, lo:hi], u_u, v_u[:, lo:hi], u_d[lo:hi, :], v_d


def shard_partial(x, shard) -> np.ndarray:
    """Rank-local [M, r_d] fp32 contribution h_p . u_down_p."""
    u_g, v_g, u_u, v_u, u_d, _ = shard
    return fused_gate_up(x, u_g, v_g, u_u, v_u) @ _f32(u_d)


def tp_finish(partial_sum, v_down) -> np.ndarray:
    return _f32(partial_sum) @ _f32(v_down)


# ---------------------------------------------------------------- metrics
def error_metrics(got, ref) -> dict:
    """rel-Frobenius, max-abs / RMS(ref) and non-finite count, the
    north-star criterion (rel <= 5e-3, max-abs <= 2e-2 * RMS), as in
    bench/checkpoint_speedup.py:20-31 and bench/all_mlp_layers.py:181-221."""
    got = _f32(got).astype(np.float64)
    ref = _f32(ref).astype(np.float64)
    diff = got - ref
    ref_norm = max(float(np.linalg.norm(ref)), 1e-30)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    return {
        "rel_fro": float(np.linalg.norm(diff)) / ref_norm,
        "max_abs": float(np.max(np.abs(diff))) if diff.size else 0.0,
        "rms": rms,
        "max_abs_over_rms": (float(np.max(np.abs(diff))) / rms) if rms > 0 else 0.0,
        "nonfinite": int(np.size(got) - np.count_nonzero(np.isfinite(got))),
    }


def within_tolerance(m: dict, rel: float = 5e-3, max_abs_rms: float = 2e-2) -> bool:
    return m["nonfinite"] == 0 and m["rel_fro"] <= rel and m["max_abs_over_rms"] <= max_abs_rms


# ------------------------------------------------------------------ inputs
def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even) and return it as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    nan = np.isnan(a)
    out = (rounded << 16).astype(np.uint32).view(np.float32)
    return np.where(nan, np.float32(np.nan), out).astype(np.float32)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns of an array already on the bf16 grid."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def make_inputs(seed: int, m: int, d: int, ff: int, r_gu: int, r_d: int | None = None):
    """Seeded inputs on the bf16 grid (returned as fp32):
    x ~ N(0,1); u (in x r) ~ N(0, 1/in); v (r x out) ~ N(0, 1/r)
    (test_speedup.py:803-808; bench/latency.py:58-72)."""
    r_d = r_gu if r_d is None else r_d
    rng = np.random.default_rng(seed)

    def mat(rows, cols):
        return bf16_round(rng.standard_normal((rows, cols), dtype=np.float32) / np.float32(np.sqrt(rows)))

    x = bf16_round(rng.standard_normal((m, d), dtype=np.float32))
    factors = (mat(d, r_gu), mat(r_gu, ff), mat(d, r_gu), mat(r_gu, ff), mat(ff, r_d), mat(r_d, d))
    return x, factors


def make_dense(seed: int, d: int, ff: int):
    """Dense weights ~ N(0, 1/in) on the bf16 grid (bench/latency.py:75-85)."""
    rng = np.random.default_rng(seed)

    def mat(rows, cols):
        return bf16_round(rng.standard_normal((rows, cols), dtype=np.float32) / np.float32(np.sqrt(rows)))

    return mat(d, ff), mat(d, ff), mat(ff, d)
