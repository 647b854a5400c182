"""CPU oracle for the block-scaled FP4 grouped GEMM -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package, and only as the checker (or the timed CPU
baseline); the product path in ratchet_b200/ never routes through it.

Modules:
  nvfp4  NVFP4 formats (E2M1 codes, E4M3 block scales, fp32 global scale),
         the quantisation recipe and the grouped dequantise-then-matmul.
  mx     the reference operator's MXFP8 x MXFP4 semantics
         (kernels/gemm/fp4_grouped_gemm/b200/kernel.py:14-26) and its host
         scale repack (kernel.py:1006-1018, :2679-2786).

Parity pins: the E2M1 rounding is checked against fixtures produced by the
reference evaluator's own FP4 cast, and the MX scale repack against fixtures
produced by the reference kernel module's host functions (tests/golden/).
"""
