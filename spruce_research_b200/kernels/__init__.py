"""Attention drop-ins mirroring the reference's kernels/ package."""
