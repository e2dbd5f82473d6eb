"""dart_cuda_b200 — B200 (sm_100a) implementation of G-Tensor's AFT-full
training hot path, exported through the reference's C ABI (libmat_mul.so).

* ``dart_cuda_b200.ops``     — PyTorch-facing calls of the batched dc_* ABI.
* ``dart_cuda_b200.gtensor`` — mirror of the reference's Python Tensor API
  (python/dart_cuda/core/tensor/gpu_tensor.py) over the handle ABI.
* ``dart_cuda_b200.build``   — nvcc build of lib/libmat_mul.so.
"""
from ._lib import LIB_PATH, DcError, check, lib  # noqa: F401

__version__ = "0.1.0"
