"""jax4j_b200: a B200-native (sm_100a) engine behind JAX4J's engine SPI.

The product is libjax4j_b200.so (C ABI in include/jax4j_b200.h). This package holds its build
recipe (build.py), the ctypes binding (_lib.py) and B200Backend (backend.py), the Python mirror
of the reference's ComputeBackend/QuantizedOps SPI.
"""
from ._lib import (OP, OPS, Q2_0, Q4_0, Q4_K, Q6_K, Q8_0, QUANT_BLOCK, QUANT_NAMES,  # noqa: F401
                   diagnostics, exported_symbols, load)

__all__ = ["OP", "OPS", "Q2_0", "Q4_0", "Q4_K", "Q6_K", "Q8_0", "QUANT_BLOCK", "QUANT_NAMES",
           "diagnostics", "exported_symbols", "load"]
