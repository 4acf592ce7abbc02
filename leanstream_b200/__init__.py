"""B200-native sparse streaming-MLP compute backend for LeanStream.

The product is the sm_100a library libleanstream_b200.so (C ABI in
include/leanstream_b200.h). This package is the Python host-side mirror of
the reference's native-backend API, plus the seeded synthetic data format.
"""
from ._native import load as load_library, LIBRARY  # noqa: F401
from .backend import B200Backend, DeviceQueue, ExecutionQueue, quantize_io_load  # noqa: F401
from .batch import BatchMLP, union_plan  # noqa: F401

__all__ = ["B200Backend", "BatchMLP", "DeviceQueue", "ExecutionQueue", "quantize_io_load", "union_plan",
           "load_library", "LIBRARY"]
