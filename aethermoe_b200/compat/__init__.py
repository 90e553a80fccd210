"""Compatibility surfaces for callers written against the reference.

``aethermoe_b200/compat`` on ``sys.path`` makes ``import mlx.core as mx``
resolve to a small NumPy-backed array module with the subset of MLX the
reference's tests and benchmarks use; the kernels themselves come from
``aethermoe_b200.kernels``.
"""
