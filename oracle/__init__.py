"""CPU oracle for the klab small-batch projection path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's CPU-side algorithms for the
hot path: BF16 round-to-nearest-even from FP64 and the tolerance check
(projection_accuracy.py), the lossless BF16 codec v1 (compressed_bf16.py,
docs/bf16-format.md), the INT8 / FP4 quantizers and dequantizers (int8_weights.py,
fp4.py) plus the benchmark's per-row INT8 and FP16-scale FP4 variants, and FP64
reference projections. Each function names the reference file:line it follows.

Parity is pinned: tests/test_oracle_golden.py checks every function here against
fixtures produced by the reference's own code (tests/golden/make_golden.py) and
against the reference's literal known-answer vectors.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
may import this package, and only as the checker or the timed CPU baseline. The
product path (klab_b200) never imports it and has no CPU fallback.
"""
