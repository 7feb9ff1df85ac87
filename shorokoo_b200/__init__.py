"""shorokoo_b200: B200-native inference backend for Shorokoo (the Shorokoo.LinuxGPU slot).

The work happens in libshorokoo_b200.so (C++/CUDA for sm_100a) behind the C ABI in
include/shorokoo_b200.h; ``backend`` mirrors the reference's plugin interface on top of it.
"""
from .backend import (  # noqa: F401
    B200ArgumentError,
    B200InferenceSession,
    B200InferenceSessionFactory,
    B200InvalidOperationError,
    B200NotSupportedError,
    B200OutOfMemoryError,
    B200TensorValue,
    ShorokooB200Error,
    ShorokooGraphOptimization,
    ShorokooLogSeverity,
    ShorokooOnnxValueType,
    ShorokooTensorElementType,
)
