"""hyperkernel_b200 — B200-native (sm_100a) continuous-batching decode step.

The product is libhk.so (include/hk.h): CUDA kernels for pack, KV append, ragged paged
attention with split-KV LSE merge, FP8 block-scaled linear and MoE, behind a C ABI that
mirrors the reference engine's `Kernel` boundary.  This Python package is a thin host
layer (ctypes) used by the tests and the benchmark; torch supplies device memory and
streams only.
"""
from . import _lib
from ._lib import HKError, check_errors, device_info, lib, version

__all__ = ["HKError", "check_errors", "device_info", "lib", "version", "_lib"]
