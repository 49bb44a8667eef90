"""lookatmyquant_b200 — LookAtMyQuant's quantization-build hot path on B200 (sm_100a).

The host side mirrors the reference's Python interfaces for the path (`opgraph.codes` → codes, `opgraph.frame` → frame,
`opgraph.syntax.sweep` → syntax, `opgraph.ldlq_gpu` → ldlq_gpu, the statistics, QEP, row-plan build, packed artifact
and KL probe of quantize.py / compiler.py → hessian, linalg, layer, artifact, kl, measure); the compute runs in
liblamq_b200.so, hand-written CUDA kernels behind a C ABI (include/lamq_b200.h).
"""

__version__ = "0.1.0"
