"""Batch-sharded block-stack harness for the krsi_b200 kernels."""
