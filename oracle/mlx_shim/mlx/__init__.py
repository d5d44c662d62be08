"""Minimal stand-in for Apple's ``mlx`` package, backed by torch on the CPU.

TEST INFRASTRUCTURE ONLY. MLX cannot be installed in this environment, so this
shim lets the reference implementation's own unmodified Python modules
(``rfsn_v10_5.cache``, ``block_manager``, ``residency``, ``attention_exact``,
``layer``, ``model``) run here, to generate golden vectors and to pin the
oracle. Only the subset of ``mlx.core`` / ``mlx.nn`` / ``mlx.utils`` that those
modules and their tests touch is provided. Arithmetic is float32 torch on the
CPU; MLX's own kernels (notably ``mx.fast.scaled_dot_product_attention``) are
replaced by their textbook definitions, so absolute floating-point values are
not MLX's — the control flow (ring indices, seal boundaries, page tables,
residency decisions) is the reference's own code.
"""
