"""CPU oracle for the exact segmented-attention path (TEST INFRASTRUCTURE).

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it. It restates, in numpy (float32 arithmetic, integer ring/page-table
logic in plain Python), the algorithms of the reference implementation
(rfsn-MLX, package ``rfsn_v10_5``); every function cites the reference
``file:line`` it follows.

Pinning: the restatement is checked against golden vectors in
``tests/golden/`` that were produced by running the reference's own unmodified
modules over ``oracle/mlx_shim`` (a torch-CPU stand-in for ``mlx``, which
cannot be installed here). Ring positions, seal boundaries, page tables and
residency decisions are therefore pinned to the reference's code; absolute
floating-point values are pinned to the reference's formulas evaluated in
float32 (MLX's own kernels, e.g. ``mx.fast.scaled_dot_product_attention``, are
not available to compare against).
"""
