"""freeml_b200 -- a B200-native (sm_100a) backend for FreeML's NanoLLM token loop.

The compute lives in libfreeml_cuda.so (CUDA kernels behind the C ABI of
include/freeml_cuda.h).  This package holds the Python host side:

  _lib        ctypes bindings (raise if the library is missing; no CPU path)
  matrix_ops  the FreeML operator names (Mul, LayerNormOp, Softmax, ...) on
              torch CUDA tensors, for the per-operator parity tests
  lm          NanoLM: the KV-cached batched greedy decode engine
  build       nvcc build of the library
"""
from ._lib import FmlError, load  # noqa: F401

__all__ = ["FmlError", "load"]
