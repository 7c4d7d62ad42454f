"""tierstream on B200: the weight-streaming runtime's C ABI (libtierstream.so) and its Python handles.

The runtime itself is native: C++ for the host control plane (descriptor, planner, slot cache, service thread) and
CUDA for sm_100a for the data path (land / write-back / compaction / peer copies, device-gated control kernels,
device xxh64). This package only locates and describes it; see abi.py for the ctypes view and runtime.py for handles.
"""
from . import abi  # noqa: F401

__all__ = ["abi"]
