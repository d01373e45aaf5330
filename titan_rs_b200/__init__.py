"""titan_rs_b200: the titan.rs operator hot path (row softmax, GEMM, attention,
conv2d) as hand-written sm_100a kernels behind the titan.rs HAL, Kernel ABI and
OpRequest contracts.

The native library (libtitan_b200.so, C ABI in include/titan_b200.h) does the
work; this package is the Python host mirror used by tests and the benchmark.
"""
from .kernel_abi import DType, KernelAbi  # noqa: F401
from .hal import HalError, Session, driver_available, enumerate_devices, last_candidate, launch_count  # noqa: F401
from .runtime import (ExecutionError, OpRequest, Runtime, TensorHandle, TensorSpec,  # noqa: F401
                      bf16_bits_to_f32, f32_to_bf16_bits, fill_normal, fill_uniform)

__all__ = ["DType", "KernelAbi", "HalError", "Session", "driver_available", "enumerate_devices", "last_candidate",
           "launch_count",
           "ExecutionError",
           "OpRequest", "Runtime", "TensorHandle", "TensorSpec", "bf16_bits_to_f32", "f32_to_bf16_bits",
           "fill_normal", "fill_uniform"]
