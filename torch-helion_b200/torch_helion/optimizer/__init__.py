"""Optimizer: canonicalisation passes, partitioning into kernels, planning."""
