"""rustyllm_b200: B200-native (sm_100a) quantized-linear hot path for rustyllm.

The compute lives in librq.so (hand-written CUDA behind the C ABI of
include/rq.h); this package is the host-side mirror of the reference's API.
"""
from ._lib import Q2_K, Q3_K, Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, RqError, lib
from .linear import Context, ParallelQ4Linear, QMatMul, QTensor, QWeight

__all__ = ["Q2_K", "Q3_K", "Q4_0", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "RqError", "lib", "Context", "ParallelQ4Linear", "QMatMul",
           "QTensor", "QWeight"]
