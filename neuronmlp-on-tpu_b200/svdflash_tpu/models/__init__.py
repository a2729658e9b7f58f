"""svdflash_tpu.models on B200."""
