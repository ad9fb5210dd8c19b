"""Independent numpy restatement of MLX affine quantization (test infrastructure).

Written separately from nq_oracle.c (vectorised over groups instead of looping)
so that the two can be checked against each other; both follow MLX's CPU
semantics for mx::quantize / mx::dequantize / mx::quantized_matmul as called at
compute/src/compute/model/mlx_ops.h:39 and
compute/src/compute/model/llama_model.cpp:67.  All fp32 arithmetic below is
numpy float32 (IEEE single, round-to-nearest-even), matching the C oracle.
"""
import numpy as np

from .oracle import bf16_to_f32, f32_to_bf16


def quantize(w, bits=4, group_size=64, scheme=0):
    w = np.asarray(w)
    wf = bf16_to_f32(w) if w.dtype == np.uint16 else w.astype(np.float32)
    rows, K = wf.shape
    g = wf.reshape(rows, K // group_size, group_size)
    n_bins = np.float32((1 << bits) - 1)
    w_max = g.max(axis=-1, keepdims=True)
    w_min = g.min(axis=-1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        if scheme == 0:
            mask = np.abs(w_min) > np.abs(w_max)
            scale = np.maximum((w_max - w_min) / n_bins, np.float32(1e-7))
            scale = np.where(mask, scale, -scale).astype(np.float32)
            edge = np.where(mask, w_min, w_max).astype(np.float32)
            q0 = np.rint(edge / scale).astype(np.float32)
            nz = q0 != 0
            scale = np.where(nz, edge / np.where(nz, q0, 1), scale).astype(np.float32)
            bias = np.where(nz, edge, np.float32(0)).astype(np.float32)
        else:
            scale = ((w_max - w_min) / n_bins).astype(np.float32)
            bias = w_min.astype(np.float32)
        q = np.rint((g - bias) / scale)
        q = np.clip(q, 0, n_bins)
        q = np.where(scale == 0, 0, q)
    q = q.astype(np.uint32).reshape(rows, K)
    per = 32 // bits
    q = q.reshape(rows, K // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    wq = np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)
    return wq, f32_to_bf16(scale[..., 0]), f32_to_bf16(bias[..., 0])


def unpack(wq, bits):
    per = 32 // bits
    shifts = np.arange(per, dtype=np.uint32) * bits
    q = (wq[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(*wq.shape[:-1], wq.shape[-1] * per)


def dequantize_f32(wq, scales, biases, bits=4, group_size=64):
    """MLX CPU dequantize: bf16(bf16(s*q) + b), returned as float32 values."""
    q = unpack(np.asarray(wq, np.uint32), bits).astype(np.float32)
    rows, K = q.shape
    s = np.repeat(bf16_to_f32(scales), group_size, axis=-1).reshape(rows, K)
    b = np.repeat(bf16_to_f32(biases), group_size, axis=-1).reshape(rows, K)
    p = bf16_to_f32(f32_to_bf16(s * q))
    return bf16_to_f32(f32_to_bf16(p + b))


def dequantize(wq, scales, biases, bits=4, group_size=64):
    return f32_to_bf16(dequantize_f32(wq, scales, biases, bits, group_size))


def qmm_f64(x, wq, scales, biases, bits=4, group_size=64):
    """Reference sums: x (bf16 bits) . w_hat^T in float64."""
    wh = dequantize_f32(wq, scales, biases, bits, group_size).astype(np.float64)
    return bf16_to_f32(x).astype(np.float64) @ wh.T
