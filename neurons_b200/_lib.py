"""Loader for libnq.so, the C-ABI library built from neurons_b200/csrc.

The library is loaded from this package directory only (never from a system
path), and loading fails loudly: there is no CPU fallback for any operation.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnq.so")

_lib = None

# nq_status (include/nq.h), mirroring compute::ErrorCode
NQ_SUCCESS = 0
STATUS_NAMES = {
    0: "Success", 1: "InvalidInput", 2: "InvalidModel", 3: "BackendNotAvailable",
    4: "ComputeError", 5: "UnknownError",
}

# exported symbol -> (restype, argtypes); the full surface of include/nq.h
P, I64, I, U64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
SIGNATURES = {
    "nq_version": (I, []),
    "nq_last_error": (ctypes.c_char_p, []),
    "nq_device_count": (I, []),
    "nq_take_device_error": (I, [P]),
    "nq_bits_from_shapes": (I, [I64, I64, I]),
    "nq_quantize": (I, [P, I, I64, I64, I, I, I, P, P, P, P]),
    "nq_dequantize": (I, [P, P, P, I64, I64, I, I, P, P]),
    "nq_dequantize_f16": (I, [P, P, P, I64, I64, I, I, P, P]),
    "nq_quantized_matmul_f16": (I, [P, I64, P, P, P, I64, I64, I, I, P, P]),
    "nq_quantized_matmul": (I, [P, I64, P, P, P, I64, I64, I, I, P, P]),
    "nq_quantized_matmul_launches": (I, [I64, I64, I64, I, I]),
    "nq_gather_qmm": (I, [P, I64, I64, P, P, I64, P, P, P, I64, I64, I64, I, I, P, P]),
    "nq_moe_route": (I, [P, I64, I64, I64, P, P, P]),
    "nq_moe_workspace_size": (U64, [I64, I64, I64, I64, I64]),
    "nq_moe_switch": (I, [P, I64, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P, P, I, I, P,
                          U64, P, P]),
    "nq_moe_switch_static": (I, [P, I64, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P, P, I,
                                 I, P, P]),
    "nq_moe_partial_workspace_size": (U64, [I64, I64, I64, I64, I64, I64]),
    "nq_quantized_matmul_push": (I, [P, I64, P, P, P, I64, I64, I, I, I64, I64, P, P]),
    "nq_quantized_matmul_push_check": (I, [P, I64, P, P, P, I64, I64, I, I, I64, I64, P]),
    "nq_moe_switch_partial": (I, [P, I64, I64, I64, I64, I64, P, P, I64, I64, P, P, P, P, P, P, P,
                                  P, P, I, I, P, U64, P, P]),
    "nq_moe_switch_partial_push": (I, [P, I64, I64, I64, I64, I64, P, P, I64, I64, P, P, P, P, P, P,
                                       P, P, P, I, I, P, U64, P, P]),
    "nq_llama_create": (I, [P, P, P, P, P, P]),
    "nq_llama_destroy": (I, [P]),
    "nq_llama_position": (I64, [P]),
    "nq_llama_reset": (I, [P, P]),
    "nq_llama_step": (I, [P, P, P, P, P]),
    "nq_llama_prefill": (I, [P, P, I64, P, P]),
    "nq_llama_generate": (I, [P, P, I64, P, P]),
}


class NQError(RuntimeError):
    """A non-success nq_status; .status holds the code, .code its ErrorCode name."""

    def __init__(self, status, message):
        self.status = status
        self.code = STATUS_NAMES.get(status, "UnknownError")
        super().__init__(f"{self.code}: {message}")


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"neurons_b200: {LIB_PATH} is missing -- build it with "
                "`python -m neurons_b200.build` (there is no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status):
    if status != NQ_SUCCESS:
        msg = lib().nq_last_error()
        raise NQError(status, msg.decode() if msg else "")
    return status
