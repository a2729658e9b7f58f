"""svdflash_b200: B200 (sm_100a) SVD-compressed LLaMA MLP hot path.

A from-scratch Blackwell implementation of the operators of
n-paradigm/NeuronMLP-on-TPU's ``svdflash_tpu`` package: the fused low-rank
gate/up operator and the XUV down operator, behind the reference's operator
names (``svdflash_b200.kernels.ops``), its model hook
(``svdflash_b200.models``) and a C ABI (``include/svdmlp.h``).
"""
from . import _lib  # noqa: F401

__version__ = "0.1.0"
