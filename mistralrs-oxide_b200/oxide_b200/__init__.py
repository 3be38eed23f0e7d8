"""oxide_b200: B200 (sm_100a) kernels for mistralrs-oxide's tensor-op hot path.

``ops`` mirrors the reference's ``src/ops`` free functions on CUDA tensors,
``backend`` mirrors ``src/cuda_backend`` (CudaBackend / KernelManager), ``pipe``
runs ops on host buffers with overlapped copies, ``dist`` holds the
row-partition and cross-GPU reduction helpers, and ``workloads`` the seeded
benchmark configurations.  All compute goes through liboxide_b200.so.
"""
from ._lib import LIB_PATH, OxideError, lib  # noqa: F401

__version__ = "0.1.0"
