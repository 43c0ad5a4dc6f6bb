"""axion_b200 — B200-native (sm_100a) Q8_0 linear hot path of the Axion runtime.

The CUDA kernels and the C ABI live in ``libaxq8.so`` (declared in
``include/axq8.h``); :mod:`axion_b200.ops` exposes them under the reference's
operator names, :mod:`axion_b200.gguf` reads/writes GGUF files.
"""
from ._lib import AxionCudaError, lib_path, load  # noqa: F401

__all__ = ["AxionCudaError", "lib_path", "load"]
