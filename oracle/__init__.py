"""TEST INFRASTRUCTURE ONLY — the CPU oracle for the quantization-build hot path.

This package restates, on the CPU, the reference algorithms that the CUDA kernels of `lookatmyquant_b200` replace
(ShinMegamiBoson/lookatmyquant: `opgraph/codes.py`, `opgraph/syntax.py`, `opgraph/frame.py`, `quantize.py`,
`compiler_artifact.py`). It is the checker for parity tests, `__graft_entry__.smoke()` and the CPU-baseline leg of
`bench.py`; the product never imports it. Each function cites the reference lines it follows.

The oracle is pinned against golden vectors produced by running the reference itself (`tests/golden/make_golden.py`,
committed with its outputs): Viterbi paths, row-trellis LDLQ words, the LDL factor, Hadamard rotations and packed bytes
all match bit-for-bit or to fp64 rounding. The Hessian accumulation and the KL reduction are inline expressions in the
reference (no callable function), so those two are pinned only by restating the expressions (fp32 GEMM / log-softmax).
"""
