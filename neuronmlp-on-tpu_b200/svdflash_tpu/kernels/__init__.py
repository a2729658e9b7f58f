"""svdflash_tpu.kernels on B200: config, pallas_ops and reference."""
