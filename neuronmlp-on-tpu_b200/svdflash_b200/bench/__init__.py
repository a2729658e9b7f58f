"""B200 ports of the reference's benchmark drivers (bench/*.py): the same
command-line flags and JSON report keys, driving the sm_100a operators
through the ``svdflash_tpu`` import facade."""
