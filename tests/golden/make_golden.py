"""Generates the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is available:
    python tests/golden/make_golden.py /path/to/NeuronMLP-on-TPU
It imports the reference's own kernels/reference.py (NumPy only), runs its
golden operators on seeded bf16-grid inputs and writes one compressed .npz
per case.  Small cases store the inputs (uint16 bf16 bit patterns) and the
full fp32 outputs.  Large cases store a SHA-256 of the inputs (the tests
regenerate them from the seed with oracle.make_inputs and check the hash)
plus the first rows and the Frobenius norm of each output, which keeps the
committed fixtures small.  The tests only read these files; they never need
the reference checkout.

Shapes are the reference tests' tail shapes (S, H, R, I) plus a few small
extra cases (tests_test_speedup_migration.py.before:47-71 in the reference).
"""
from __future__ import annotations

import importlib.util
import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import svdmlp_oracle as orc  # noqa: E402

CASES = [
    # name, seed, S, H, R, I
    ("tail_1_129_131_137", 11, 1, 129, 131, 137),
    ("tail_129_257_257_513", 12, 129, 257, 257, 513),
    ("tiles_257_513_513_1025", 13, 257, 513, 513, 1025),
    ("dense_tail_3_257_1025_513", 14, 3, 257, 1025, 513),
    ("small_8_64_40_96", 15, 8, 64, 40, 96),
]


def input_digest(inputs: dict) -> str:
    """SHA-256 over the bf16 bit patterns of the inputs, in sorted-name order."""
    import hashlib
    h = hashlib.sha256()
    for k in sorted(inputs):
        h.update(k.encode())
        h.update(orc.bf16_bits(inputs[k]).tobytes())
    return h.hexdigest()


def load_reference(root: pathlib.Path):
    spec = importlib.util.spec_from_file_location("ref_kernels_reference", root / "kernels" / "reference.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(root: str) -> None:
    ref = load_reference(pathlib.Path(root))
    index = {}
    for name, seed, s, h, r, i in CASES:
        x, f = orc.make_inputs(seed, s, h, i, r)
        wg, wu, wd = orc.make_dense(seed + 1000, h, i)
        # fp32 arrays on the bf16 grid: the reference computes in fp32 and
        # never rounds an intermediate (its .astype(x.dtype) is fp32 here).
        gate_up = ref.fused_gate_up_ref(x, f[0], f[1], f[2], f[3])
        xuv = ref.fused_xuv_ref(gate_up, f[4], f[5])
        full = ref.svd_mlp_ref(x, *f)
        dense = ref.dense_mlp_ref(x, wg, wu, wd)
        silu_in = np.linspace(-30, 30, 241, dtype=np.float32)
        inputs = dict(x=x, u_gate=f[0], v_gate=f[1], u_up=f[2], v_up=f[3], u_down=f[4], v_down=f[5],
                      w_gate=wg, w_up=wu, w_down=wd)
        outputs = dict(gate_up=gate_up, xuv=xuv, svd_mlp=full, dense_mlp=dense)
        n_in = sum(a.size for a in inputs.values())
        payload = dict(silu_in=silu_in, silu_out=ref.silu(silu_in).astype(np.float32))
        full_case = n_in <= 400_000
        if full_case:
            payload.update({k: orc.bf16_bits(v) for k, v in inputs.items()})
            payload.update({k: v.astype(np.float32) for k, v in outputs.items()})
        else:
            payload["inputs_sha256"] = np.frombuffer(input_digest(inputs).encode(), dtype=np.uint8)
            for k, v in outputs.items():
                payload[k + "_head"] = v[:8].astype(np.float32)
                payload[k + "_norm"] = np.float64(np.linalg.norm(v.astype(np.float64)))
        np.savez_compressed(HERE / f"{name}.npz", **payload)
        index[name] = {"seed": seed, "S": s, "H": h, "R": r, "I": i, "full": full_case}
    index["low_rank_dim"] = {f"{h}_{i}_{c}": ref.low_rank_dim(h, i, c)
                             for h, i in ((4096, 14336), (3072, 8192), (2048, 8192), (8192, 28672))
                             for c in (0.4, 0.6, 0.8, 0.9)}
    (HERE / "index.json").write_text(json.dumps(index, indent=1, sort_keys=True) + "\n")
    print(json.dumps(index["low_rank_dim"]))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python make_golden.py <path to the reference checkout>")
    main(sys.argv[1])
