"""B200-native (sm_100a) implementation of ZeroLlm's quantized-linear + paged-KV decode path.

The product is libzero_tensor.so (zeroplatform_b200/csrc, C ABI in include/); this package is the
Python host mirror of the reference operators used by the tests and the benchmark.
"""
from ._lib import ZcError, lib  # noqa: F401

__version__ = "0.1.0"
