"""TensorOperations-B200: a B200-native (sm_100a) evaluator for the fused
spectral-element stiffness path of Rohit-Kakodkar/TensorOperations.

The product is the C ABI in include/tensoroperations_b200.h (implemented by
libtensoroperations_b200.so, built from csrc/) and the header-only C++
frontend; this Python package is the ctypes binding used by the tests and the
benchmark driver.
"""
from . import abi  # noqa: F401  (loads the library; ImportError if it is not built)

__all__ = ["abi"]
