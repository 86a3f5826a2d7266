"""Data-parallel communication: ring algorithm, sparsifier, membership and NVLink kernels."""
