"""CPU oracle for the Flash-Next sparse-MoE decode path -- TEST INFRASTRUCTURE ONLY.

This package is a NumPy restatement of the reference's arithmetic for the hot
path (router, top-k, renorm, Q4/G32 affine projections, bfloat16 SwiGLU,
slot-ordered weighted combine, shared expert, token grouping, paged decode
attention).  It exists to check the CUDA path, never to stand in for it:

* only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
  leg may import it;
* the product package (``flashnext_b200``) never imports it and fails loudly
  when its CUDA library is missing.

Every function cites the reference file:line it follows.  Where the reference
leaves an arithmetic detail to a library that is absent here (MLX 0.32.2 and
mlx-vlm 0.6.17 are not installed and cannot be), the oracle fixes one
documented, deterministic choice and the CUDA kernels implement the same one,
so the two agree bit for bit.  Pinning: the Q4 decode formula, the executor's
reference path and ``weighted_combine`` are checked against outputs of the
reference's own NumPy code (``tests/golden``); the MLX-level pieces (router
softmax/top-k, bfloat16 SwiGLU sequence, attention) are unpinned against MLX.
"""
