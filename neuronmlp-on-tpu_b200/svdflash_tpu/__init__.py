"""Import-compatible facade of the reference's ``svdflash_tpu`` package.

The reference's benches and model import ``svdflash_tpu.kernels.config``,
``svdflash_tpu.kernels.pallas_ops``, ``svdflash_tpu.kernels.reference``,
``svdflash_tpu.models.hf_svd`` and ``svdflash_tpu.test_speedup``
(bench/latency.py:23-42, bench/speedup.py:20-31, bench/all_mlp_layers.py:21-31,
bench/e2e_block.py:40-48, bench/tune.py:20-27, models/modeling_llama.py:62-73).
Each module here re-exports the same names from ``svdflash_b200``, whose
operators run only on the sm_100a library: a caller that switches its
import root to this package drives the B200 kernels.  Arrays are torch CUDA
tensors instead of jax arrays (``kernels.reference`` also takes NumPy).
"""
