"""lookatmyquant_b200 — LookAtMyQuant's quantization-build hot path on B200 (sm_100a).

The host side mirrors the reference's Python interfaces (`opgraph.codes`, `opgraph.frame`); the compute runs in
liblamq_b200.so, hand-written CUDA kernels behind a C ABI (include/lamq_b200.h).
"""

__version__ = "0.1.0"
