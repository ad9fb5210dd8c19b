"""neurons_b200 -- B200 (sm_100a) implementation of neurons' MLX-affine
quantized-matmul path, behind a C ABI (include/nq.h, libnq.so).

The package holds the CUDA kernels and the C ABI (csrc/), the C++ backend
(CUDABackend behind the ComputeBackend interface, csrc/cuda_backend.*) and
this Python mirror of the MLX entry points the reference calls (ops.py),
the tensor/expert-parallel sharding over NCCL (dist.py, libnq_dist.so) and
a decode-step replay of LlamaModel's quantized linears (replay.py).
"""
from ._lib import LIB_PATH, NQError, lib
from .ops import (SCHEME_MINMAX, SCHEME_MLX_AFFINE, bits, dequantize, gather_qmm, lin,
                  moe_partial_workspace_size, moe_route, moe_switch, moe_switch_partial,
                  moe_workspace_size, quantize, quantized_matmul, quantized_matmul_launches,
                  take_device_error)

__all__ = [
    "LIB_PATH", "NQError", "lib", "SCHEME_MINMAX", "SCHEME_MLX_AFFINE", "bits", "dequantize",
    "gather_qmm", "lin", "moe_partial_workspace_size", "moe_route", "moe_switch",
    "moe_switch_partial", "moe_workspace_size", "quantize",
    "quantized_matmul", "quantized_matmul_launches", "take_device_error",
]
