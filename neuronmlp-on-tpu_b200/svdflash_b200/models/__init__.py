"""Model hooks: the SVD / dense LLaMA MLP modules and the MLP-only block stack."""
from .svd_mlp import DenseLlamaMLP, MlpBlockStack, SvdLlamaMLP  # noqa: F401
