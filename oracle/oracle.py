"""ctypes front end of the C oracle (oracle/nq_oracle.c) -- test infrastructure.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module.  bf16 tensors are passed as numpy uint16 arrays holding the raw
bf16 bit patterns; packed codes as uint32; indices as int32.
"""
import ctypes

import numpy as np

from . import build as _build

_lib = None

SCHEME_MLX = 0      # MLX affine quantizer (edge snapping)
SCHEME_MINMAX = 1   # scale=(max-min)/n_bins, bias=min


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        _lib = ctypes.CDLL(path)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        _lib.or_f32_to_bf16.restype = ctypes.c_uint16
        _lib.or_f32_to_bf16.argtypes = [ctypes.c_float]
        _lib.or_bf16_to_f32.restype = ctypes.c_float
        _lib.or_bf16_to_f32.argtypes = [ctypes.c_uint16]
        _lib.or_bits_from_shapes.argtypes = [I64, I64, I]
        _lib.or_quantize.argtypes = [P, I, I64, I64, I, I, I, P, P, P]
        _lib.or_dequantize.argtypes = [P, P, P, I64, I64, I, I, P]
        _lib.or_qmm.argtypes = [P, I64, P, P, P, I64, I64, I, I, P, P, I]
        _lib.or_gather_qmm.argtypes = [P, I64, I64, P, P, I64, P, P, P, I64, I64, I64,
                                       I, I, P, P, I]
        _lib.or_moe_route.argtypes = [P, I64, I64, I64, P, P]
        _lib.or_moe_switch.argtypes = [P, I64, I64, I64, I64, I64, P, P,
                                       P, P, P, P, P, P, P, P, P, I, I, I, P, I]
        _lib.or_moe_hidden.argtypes = [P, I64, I64, I64, I64, I64, P, P, P, P, P, P, P,
                                       I, I, I, P, I]
        _lib.or_moe_combine.argtypes = [P, I64, I64, I64, I64, I64, P, P, P, P, P,
                                        I, I, I, P, I]
        _lib.or_max_threads.argtypes = []
        _lib.or_f32_to_f16.restype = ctypes.c_uint16
        _lib.or_f32_to_f16.argtypes = [ctypes.c_float]
        _lib.or_f16_to_f32.restype = ctypes.c_float
        _lib.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        _lib.or_dequantize_f16.argtypes = [P, P, P, I64, I64, I, I, P]
        _lib.or_qmm_f16.argtypes = [P, I64, P, P, P, I64, I64, I, I, P, P, I]
    return _lib


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _check(rc, what):
    if rc != 0:
        raise ValueError(f"oracle {what}: invalid input (status {rc})")


def max_threads() -> int:
    return lib().or_max_threads()


def bits_from_shapes(w_cols: int, s_cols: int, group_size: int) -> int:
    return lib().or_bits_from_shapes(w_cols, s_cols, group_size)


def quantize(w, bits=4, group_size=64, scheme=SCHEME_MLX, f16=False):
    """w: [rows, K] float32, bf16-bits uint16, or (f16=True) fp16-bits uint16 ->
    (wq uint32, scales u16, biases u16); fp16 weights give fp16 scales/biases."""
    w = np.ascontiguousarray(w)
    if w.dtype == np.float32:
        dt = 0
    elif w.dtype == np.uint16:
        dt = 2 if f16 else 1
    else:
        raise TypeError("w must be float32 or 16-bit bit patterns (uint16)")
    rows, K = w.shape
    wq = np.zeros((rows, K * bits // 32), np.uint32)
    s = np.zeros((rows, K // group_size), np.uint16)
    b = np.zeros((rows, K // group_size), np.uint16)
    _check(lib().or_quantize(_p(w), dt, rows, K, bits, group_size, scheme,
                             _p(wq), _p(s), _p(b)), "quantize")
    return wq, s, b


def dequantize(wq, scales, biases, bits=4, group_size=64, f16=False):
    """f16=True: fp16 scales/biases bit patterns, fp16 output."""
    wq, scales, biases = _c(wq, np.uint32), _c(scales, np.uint16), _c(biases, np.uint16)
    rows = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    out = np.zeros((rows, K), np.uint16)
    fn = lib().or_dequantize_f16 if f16 else lib().or_dequantize
    _check(fn(_p(wq), _p(scales), _p(biases), rows, K, bits, group_size, _p(out)), "dequantize")
    return out


def f32_to_f16(a):
    """fp32 -> fp16 bit patterns, round to nearest even (the oracle's C conversion)."""
    a = np.asarray(a, np.float32)
    f = lib().or_f32_to_f16
    return np.array([f(float(v)) for v in a.reshape(-1)], np.uint16).reshape(a.shape)


def f16_to_f32(h):
    return np.ascontiguousarray(h, np.uint16).view(np.float16).astype(np.float32)


def qmm(x, wq, scales, biases, bits=4, group_size=64, nthreads=0, want_f32=False, f16=False):
    """y = x . dequant(w)^T ; x [M,K] bf16 bits -> y [M,N] bf16 bits (and fp32 sums);
    f16=True: x, scales, biases and y are fp16 bit patterns."""
    x, wq = _c(x, np.uint16), _c(wq, np.uint32)
    scales, biases = _c(scales, np.uint16), _c(biases, np.uint16)
    M, K = x.shape
    N = wq.shape[0]
    y = np.zeros((M, N), np.uint16)
    y32 = np.zeros((M, N), np.float32) if want_f32 else None
    fn = lib().or_qmm_f16 if f16 else lib().or_qmm
    _check(fn(_p(x), M, _p(wq), _p(scales), _p(biases), N, K, bits,
              group_size, _p(y), _p(y32), nthreads), "qmm")
    return (y, y32) if want_f32 else y


def gather_qmm(x, wq, scales, biases, rhs, lhs=None, bits=4, group_size=64,
               nthreads=0):
    """MLX gather_qmm (transpose=true): x [B,M,K], w [E,N,Kp] -> out [n_idx,M,N]."""
    x = _c(x, np.uint16)
    if x.ndim == 2:
        x = x[None]
    wq = _c(wq, np.uint32)
    scales, biases = _c(scales, np.uint16), _c(biases, np.uint16)
    rhs = _c(rhs, np.int32).reshape(-1)
    lhs = None if lhs is None else _c(lhs, np.int32).reshape(-1)
    B, M, K = x.shape
    E, N = wq.shape[0], wq.shape[1]
    out = np.zeros((rhs.size, M, N), np.uint16)
    _check(lib().or_gather_qmm(_p(x), B, M, _p(lhs), _p(rhs), rhs.size, _p(wq),
                               _p(scales), _p(biases), E, N, K, bits, group_size,
                               _p(out), None, nthreads), "gather_qmm")
    return out


def moe_route(logits, top_k):
    logits = _c(logits, np.uint16)
    T, E = logits.shape
    idx = np.zeros((T, top_k), np.int32)
    sc = np.zeros((T, top_k), np.float32)
    _check(lib().or_moe_route(_p(logits), T, E, top_k, _p(idx), _p(sc)), "moe_route")
    return idx, sc


def moe_switch(x, idx, scores, gate, up, down, bits=4, group_size=64, rounding=1,
               nthreads=0):
    """gate/up/down: (wq, scales, biases) stacked over experts."""
    x = _c(x, np.uint16)
    idx, scores = _c(idx, np.int32), _c(scores, np.float32)
    T, H = x.shape
    top_k = idx.shape[1]
    wg, sg, bg = (_c(gate[0], np.uint32), _c(gate[1], np.uint16), _c(gate[2], np.uint16))
    wu, su, bu = (_c(up[0], np.uint32), _c(up[1], np.uint16), _c(up[2], np.uint16))
    wd, sd, bd = (_c(down[0], np.uint32), _c(down[1], np.uint16), _c(down[2], np.uint16))
    E, I = wg.shape[0], wg.shape[1]
    y = np.zeros((T, H), np.uint16)
    _check(lib().or_moe_switch(_p(x), T, H, I, E, top_k, _p(idx), _p(scores),
                               _p(wg), _p(sg), _p(bg), _p(wu), _p(su), _p(bu),
                               _p(wd), _p(sd), _p(bd), bits, group_size, rounding,
                               _p(y), nthreads), "moe_switch")
    return y


def moe_hidden(x, idx, gate, up, bits=4, group_size=64, rounding=1, nthreads=0):
    """Stage 1 of the switch step: h [T*top_k, I] bf16 bits, pair order t*top_k + j."""
    x = _c(x, np.uint16)
    idx = _c(idx, np.int32)
    T, H = x.shape
    top_k = idx.shape[1]
    wg, sg, bg = (_c(gate[0], np.uint32), _c(gate[1], np.uint16), _c(gate[2], np.uint16))
    wu, su, bu = (_c(up[0], np.uint32), _c(up[1], np.uint16), _c(up[2], np.uint16))
    E, I = wg.shape[0], wg.shape[1]
    h = np.zeros((T * top_k, I), np.uint16)
    _check(lib().or_moe_hidden(_p(x), T, H, I, E, top_k, _p(idx), _p(wg), _p(sg), _p(bg),
                               _p(wu), _p(su), _p(bu), bits, group_size, rounding, _p(h),
                               nthreads), "moe_hidden")
    return h


def moe_combine(h, idx, scores, down, bits=4, group_size=64, rounding=1, nthreads=0):
    """Stage 2 of the switch step: y [T, H] from h [T*top_k, I] (pair order)."""
    h = _c(h, np.uint16)
    idx, scores = _c(idx, np.int32), _c(scores, np.float32)
    T, top_k = idx.shape
    wd, sd, bd = (_c(down[0], np.uint32), _c(down[1], np.uint16), _c(down[2], np.uint16))
    E, H = wd.shape[0], wd.shape[1]
    I = h.shape[1]
    y = np.zeros((T, H), np.uint16)
    _check(lib().or_moe_combine(_p(h), T, H, I, E, top_k, _p(idx), _p(scores), _p(wd),
                                _p(sd), _p(bd), bits, group_size, rounding, _p(y), nthreads),
           "moe_combine")
    return y


# ---------------------------------------------------------------- bf16 helpers

def f32_to_bf16(a):
    """Round-to-nearest-even fp32 -> bf16 bits (numpy, vectorised)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h):
    h = np.ascontiguousarray(h, dtype=np.uint16)
    return (h.astype(np.uint32) << 16).view(np.float32)
