"""B200-native rebuild of MoEInfra's quantized-expert hot path.

Subpackages mirror the reference's public API (``engine``, ``model``,
``cache``, ``transfer``); the compute runs in hand-written sm_100a CUDA
kernels behind the C ABI in ``include/moe_b200.h`` (``moeinfra_b200._native``).
"""
__version__ = "0.1.0"
