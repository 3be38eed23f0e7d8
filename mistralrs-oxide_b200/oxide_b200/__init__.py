"""oxide_b200: B200 (sm_100a) kernels for mistralrs-oxide's tensor-op hot path.

``ops`` mirrors the reference's ``src/ops`` free functions on CUDA tensors,
``pipe`` runs ops on host buffers through the library's pipelined
host-buffer entry points (oxide_pipe_*), ``loading`` decodes safetensors
weights on the GPU, ``dist`` holds the row-partition and cross-GPU reduction
helpers, ``workloads`` the seeded benchmark configurations, and ``_lib`` the
ctypes binding of liboxide_b200.so, through which all compute goes.
"""
from ._lib import LIB_PATH, OxideError, lib  # noqa: F401

__version__ = "0.1.0"
