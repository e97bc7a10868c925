"""CPU oracle of the ShapeForge task operators — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (fp64), the fp64 reference of every task operator the B200
backend implements, each function citing the reference file:line it follows.  It is the
checker the parity tests compare the CUDA kernels against; it is pinned against the
reference's own golden vectors (the G0 corpus archives and outputs of the reference task
modules, committed under ``tests/golden/``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import this package.  The product (``shapeforge_b200``) never imports it and has no CPU
fallback.

Pinning status per operator (see ``tests/test_oracle_golden.py``):

* pinned by G0 corpus bytes: rmsnorm, softmax, reduction_sum, silu, swiglu, gemm (NN);
* pinned by reference-module outputs: bitdelta_gemm, flash_attention (non-causal), rope,
  varlen_kda (and through it the shared delta-rule core used by the gated variant), mamba2,
  relu, sigmoid, sigmoid_shift, lion (and its ``error_scale`` hook), gemv and gemm_silu;
* variants that exist only as formulas (gemm_nt, bitdelta_gemm_base, causal attention,
  varlen_kda_gated) reuse a pinned function on transformed inputs (``A @ B^T`` is the pinned
  NN product with ``B^T``; the causal mask is the pinned attention with a mask; the gated KDA
  is the pinned delta-rule core with a supplied log-decay), so their parity is pinned through
  those functions, not independently.
"""

from .dtypes import from_storage, to_storage, round_to  # noqa: F401
from . import ops  # noqa: F401
