"""Python mirror of the quantized-linear entry points, over the C ABI.

Names and argument meaning follow the MLX calls that neurons makes
(compute/src/compute/model/mlx_ops.h:20-42 and the model files):

    quantize(w, group_size, bits)                    -> (wq, scales, biases)   mx::quantize
    dequantize(wq, scales, biases, group_size, bits) -> w_hat                  mx::dequantize
    quantized_matmul(x, wq, scales, biases, transpose=True, group_size, bits)  mx::quantized_matmul
    gather_qmm(x, wq, scales, biases, lhs_indices, rhs_indices, transpose=True,
               group_size, bits)                                               mx::gather_qmm
    lin(x, key, wm, gs)                                                        mlx_ops::lin
    bits(w, s, gs)                                                             mlx_ops::bits
    moe_route(logits, top_k) / moe_switch(...)        the switch step of
                                                      qwen3_transformer_moe_model_mlx.cpp:29-79

Tensors are torch CUDA tensors (device memory and streams come from torch;
the arithmetic is libnq's): activations torch.bfloat16, packed codes
torch.uint32 (torch.int32 is accepted as the same bits), scales/biases
torch.bfloat16.  Every call is asynchronous on torch's current stream.
Errors raise NQError carrying the reference's ErrorCode name.
"""
import ctypes

import torch

from ._lib import NQError, check, lib

SCHEME_MLX_AFFINE = 0
SCHEME_MINMAX = 1

_PACKED = (torch.uint32, torch.int32)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _need(t, name, dtypes):
    if t is None:
        raise NQError(1, f"{name} is required")
    if not t.is_cuda:
        raise NQError(1, f"{name} must be a CUDA tensor")
    if t.dtype not in dtypes:
        raise NQError(1, f"{name} has dtype {t.dtype}, expected one of {dtypes}")
    if not t.is_contiguous():
        raise NQError(1, f"{name} must be contiguous")
    return t


def bits(w, s, gs):
    """mlx_ops::bits: round(32 * (w.shape[-1] / s.shape[-1]) / gs), 4 if not positive."""
    return lib().nq_bits_from_shapes(int(w.shape[-1]), int(s.shape[-1]), int(gs))


def quantize(w, group_size=64, bits=4, scheme=SCHEME_MLX_AFFINE, out=None):
    """MLX affine quantize along the last axis; out: optional (wq, scales, biases).
    Scales and biases are bf16, or fp16 for fp16 weights (MLX keeps the dtype)."""
    _need(w, "w", (torch.float32, torch.bfloat16, torch.float16))
    K = int(w.shape[-1])
    rows = w.numel() // K if K else 0
    lead = tuple(w.shape[:-1])
    sdt = torch.float16 if w.dtype == torch.float16 else torch.bfloat16
    if out is None:
        wq = torch.empty(lead + (K * bits // 32,), dtype=torch.uint32, device=w.device)
        s = torch.empty(lead + (K // group_size,), dtype=sdt, device=w.device)
        b = torch.empty_like(s)
    else:
        wq, s, b = out
        _need(wq, "wq", _PACKED)
        _need(s, "scales", (sdt,))
        _need(b, "biases", (sdt,))
    dt = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[w.dtype]
    check(lib().nq_quantize(_ptr(w), dt, rows, K, bits, group_size, scheme, _ptr(wq), _ptr(s),
                            _ptr(b), _stream()))
    return wq, s, b


def dequantize(wq, scales, biases, group_size=64, bits=4, out=None):
    """bf16 scales/biases -> bf16 weights; fp16 -> fp16 (MLX keeps the dtype)."""
    _need(wq, "w", _PACKED)
    _need(scales, "scales", (torch.bfloat16, torch.float16))
    _need(biases, "biases", (scales.dtype,))
    K = int(wq.shape[-1]) * 32 // bits
    rows = wq.numel() // int(wq.shape[-1])
    if out is None:
        out = torch.empty(tuple(wq.shape[:-1]) + (K,), dtype=scales.dtype, device=wq.device)
    fn = lib().nq_dequantize_f16 if scales.dtype == torch.float16 else lib().nq_dequantize
    check(fn(_ptr(wq), _ptr(scales), _ptr(biases), rows, K, bits, group_size, _ptr(out),
             _stream()))
    return out


def quantized_matmul(x, wq, scales, biases=None, transpose=True, group_size=64, bits=4, out=None):
    if not transpose:
        raise NQError(1, "quantized_matmul: only transpose=True (the MLX linear layout) is served")
    _need(x, "x", (torch.bfloat16, torch.float16))
    _need(wq, "w", _PACKED)
    _need(scales, "scales", (x.dtype,))
    if biases is not None:
        _need(biases, "biases", (x.dtype,))
    K = int(x.shape[-1])
    M = x.numel() // K if K else 0
    N = int(wq.shape[0])
    if int(wq.shape[-1]) * 32 // bits != K:
        raise NQError(1, f"quantized_matmul: x has K={K} but w holds "
                         f"{int(wq.shape[-1]) * 32 // bits} columns at {bits} bits")
    if out is None:
        out = torch.empty(tuple(x.shape[:-1]) + (N,), dtype=x.dtype, device=x.device)
    fn = lib().nq_quantized_matmul_f16 if x.dtype == torch.float16 else lib().nq_quantized_matmul
    check(fn(_ptr(x), M, _ptr(wq), _ptr(scales), _ptr(biases), N, K, bits, group_size,
             _ptr(out), _stream()))
    return out


def quantized_matmul_launches(M, N, K, group_size=64, bits=4):
    """Kernels one quantized_matmul of an [M, K] x [N, K]^T problem launches on the
    current device: 1, or 2 when the tensor-core grid's last wave is split."""
    n = lib().nq_quantized_matmul_launches(int(M), int(N), int(K), bits, group_size)
    check(min(n, 0))
    return n


def gather_qmm(x, wq, scales, biases, lhs_indices=None, rhs_indices=None, transpose=True,
               group_size=64, bits=4, out=None):
    """MLX gather_qmm, transpose=True: out[i] = x[xi] . dequant(w[rhs[i]])^T, shape
    [n_idx, M, N] for x [B, M, K] (or [M, K] with B = 1)."""
    if not transpose:
        raise NQError(1, "gather_qmm: only transpose=True is served")
    _need(x, "x", (torch.bfloat16,))
    _need(wq, "w", _PACKED)
    _need(scales, "scales", (torch.bfloat16,))
    _need(biases, "biases", (torch.bfloat16,))
    _need(rhs_indices, "rhs_indices", (torch.int32,))
    if lhs_indices is not None:
        _need(lhs_indices, "lhs_indices", (torch.int32,))
    K = int(x.shape[-1])
    M = int(x.shape[-2]) if x.dim() >= 2 else 1
    xb = x.numel() // (M * K)
    E, N = int(wq.shape[0]), int(wq.shape[1])
    n = rhs_indices.numel()
    if out is None:
        out = torch.empty((n, M, N), dtype=torch.bfloat16, device=x.device)
    check(lib().nq_gather_qmm(_ptr(x), xb, M, _ptr(lhs_indices), _ptr(rhs_indices), n, _ptr(wq),
                              _ptr(scales), _ptr(biases), E, N, K, bits, group_size, _ptr(out),
                              _stream()))
    return out


def lin(x, key, wm, gs, out=None):
    """mlx_ops::lin: quantized (affine) matmul if '<key>.scales' exists."""
    w = wm[key + ".weight"]
    s = wm.get(key + ".scales")
    if s is None:
        # unquantized layer: matmul(x, w^T) as mlx_ops.h:41 does (a library GEMM,
        # as in the C++ cuda_ops::lin)
        _need(x, "x", (torch.bfloat16,))
        _need(w, "w", (torch.bfloat16,))
        if out is None:
            return torch.matmul(x, w.t())
        return torch.matmul(x, w.t(), out=out)
    b = wm.get(key + ".biases")
    return quantized_matmul(x, w, s, b, True, gs, bits(w, s, gs), out=out)


def moe_route(logits, top_k):
    """Router of the switch step: softmax(fp32) over all experts, top-k, renormalised.
    Returns (indices int32 [T, k] in descending probability, scores fp32 [T, k])."""
    _need(logits, "logits", (torch.bfloat16,))
    T, E = int(logits.shape[0]), int(logits.shape[1])
    idx = torch.empty((T, top_k), dtype=torch.int32, device=logits.device)
    sc = torch.empty((T, top_k), dtype=torch.float32, device=logits.device)
    check(lib().nq_moe_route(_ptr(logits), T, E, top_k, _ptr(idx), _ptr(sc), _stream()))
    return idx, sc


def moe_workspace_size(T, E, top_k, H, I):
    return int(lib().nq_moe_workspace_size(T, E, top_k, H, I))


def moe_switch(x, idx, scores, gate, up, down, group_size=64, bits=4, workspace=None, out=None):
    """Switch-MLP for T tokens given the routing; gate/up/down are (wq, scales, biases)
    stacked over experts ([E, I, H/pack], [E, H, I/pack])."""
    _need(x, "x", (torch.bfloat16,))
    _need(idx, "idx", (torch.int32,))
    _need(scores, "scores", (torch.float32,))
    T, H = int(x.shape[0]), int(x.shape[1])
    top_k = int(idx.shape[1])
    E, I = int(gate[0].shape[0]), int(gate[0].shape[1])
    for name, t in (("gate", gate), ("up", up), ("down", down)):
        _need(t[0], name + ".weight", _PACKED)
        _need(t[1], name + ".scales", (torch.bfloat16,))
        _need(t[2], name + ".biases", (torch.bfloat16,))
    need = moe_workspace_size(T, E, top_k, H, I)
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    check(lib().nq_moe_switch(_ptr(x), T, H, I, E, top_k, _ptr(idx), _ptr(scores),
                              _ptr(gate[0]), _ptr(gate[1]), _ptr(gate[2]),
                              _ptr(up[0]), _ptr(up[1]), _ptr(up[2]),
                              _ptr(down[0]), _ptr(down[1]), _ptr(down[2]),
                              bits, group_size, _ptr(workspace), workspace.numel(), _ptr(out),
                              _stream()))
    return out


def moe_partial_workspace_size(T, E, ne, top_k, H, I):
    return int(lib().nq_moe_partial_workspace_size(T, E, ne, top_k, H, I))


def moe_switch_partial(x, idx, scores, gate, up, down, E, e0, group_size=64, bits=4,
                       workspace=None, out=None):
    """fp32 share [T, H] of the switch step that the experts [e0, e0 + ne)
    contribute; gate/up/down hold those ne experts.  Summed over all shards
    and rounded to bf16 it is moe_switch's result."""
    _need(x, "x", (torch.bfloat16,))
    T, H = int(x.shape[0]), int(x.shape[1])
    top_k = int(idx.shape[1])
    ne, I = int(gate[0].shape[0]), int(gate[0].shape[1])
    need = moe_partial_workspace_size(T, E, ne, top_k, H, I)
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=x.device)
    check(lib().nq_moe_switch_partial(_ptr(x), T, H, I, E, top_k, _ptr(idx), _ptr(scores), e0, ne,
                                      _ptr(gate[0]), _ptr(gate[1]), _ptr(gate[2]),
                                      _ptr(up[0]), _ptr(up[1]), _ptr(up[2]),
                                      _ptr(down[0]), _ptr(down[1]), _ptr(down[2]),
                                      bits, group_size, _ptr(workspace), workspace.numel(),
                                      _ptr(out), _stream()))
    return out


def take_device_error():
    v = ctypes.c_uint(0)
    check(lib().nq_take_device_error(ctypes.byref(v)))
    return v.value
