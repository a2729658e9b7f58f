"""Model hooks: the SVD / dense LLaMA MLP modules, the MLP-only block stack and
the safetensors checkpoint loader (hf_svd)."""
from . import hf_svd  # noqa: F401
from .svd_mlp import DenseLlamaMLP, MlpBlockStack, SvdLlamaMLP, SvdMlpBlock  # noqa: F401
