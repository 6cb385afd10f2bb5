"""hif4x -- B200-native NVFP4 -> HiF4 conversion engine.

The hot path is hand-written sm_100a CUDA in libhif4x.so (C ABI declared in
include/hif4x.h), reached through ctypes; torch supplies device memory,
streams and torch.distributed only.
"""
from . import _lib  # noqa: F401

__version__ = "0.1.0"
