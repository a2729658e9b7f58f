"""svdflash_tpu.models.hf_svd on B200 (see svdflash_b200.models.hf_svd)."""
from svdflash_b200.models.hf_svd import *  # noqa: F401,F403
from svdflash_b200.models.hf_svd import __all__  # noqa: F401
