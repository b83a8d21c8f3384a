"""Drop-in mirrors of slotstream_spark/kernels on the MoE hot path, backed by the sm_100a C-ABI library."""
