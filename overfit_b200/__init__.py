"""overfit_b200 — B200-native (sm_100a) quantized-projection inference path.

A drop-in for Overfit's CPU decode path (DevOnBike/Overfit,
Sources/Main/LanguageModels/Runtime): the CUDA work lives in
libovf_cuda.so behind the C ABI in include/ovf.h; this package is the thin
host mirror of the reference's kernel classes (``kernels``) and of its
engine/session interfaces (``engine``).
"""
from ._lib import OverfitCudaError, OverfitRuntimeError, load  # noqa: F401

__all__ = ["load", "OverfitRuntimeError", "OverfitCudaError"]
