"""Llama decode step on the GPU (libnq.so, nq_llama_*): the quantized
matmuls of the reference's LlamaModel decode function
(compute/src/compute/model/llama_model.cpp:355-509) with RMSNorm, RoPE, GQA
attention over a KV cache and greedy argmax around them, and its pipelined
generation (:713-812) as back-to-back steps that feed each other's token on
the device.

    dec = LlamaDecoder(cfg, weights)      # weights: torch CUDA tensors
    dec.prefill(prompt_ids)               # int32 CUDA tensor
    ids = dec.generate(64)                # int32 CUDA tensor of 64 tokens
"""
import ctypes

import torch

from . import ops
from ._lib import NQError, check, lib

P = ctypes.c_void_p


class QWeight(ctypes.Structure):
    _fields_ = [("w", P), ("scales", P), ("biases", P)]


class LlamaConfig(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("intermediate", ctypes.c_int), ("vocab", ctypes.c_int), ("bits", ctypes.c_int),
                ("group_size", ctypes.c_int), ("max_context", ctypes.c_int),
                ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)]


class LlamaLayer(ctypes.Structure):
    _fields_ = [("input_norm", P), ("post_norm", P)] + [
        (n, QWeight) for n in ("q", "k", "v", "o", "gate", "up", "down")]


CONFIG_KEYS = [f for f, _ in LlamaConfig._fields_]
PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def _qw(t):
    if t is None:
        return QWeight(None, None, None)
    w, s, b = t
    return QWeight(P(w.data_ptr()), P(s.data_ptr()) if s is not None else None,
                   P(b.data_ptr()) if b is not None else None)


class LlamaDecoder:
    """cfg: dict with the LlamaConfig fields.  weights: dict with 'embed'
    (wq, scales, biases), 'final_norm' (bf16), optional 'lm_head' (wq, s, b) and
    'layers': a list of dicts with 'input_norm', 'post_norm' and the seven
    projections as (wq, scales, biases), all CUDA tensors (kept referenced)."""

    def __init__(self, cfg, weights):
        self.cfg = dict(cfg)
        self._keep = weights
        c = LlamaConfig(**{k: self.cfg[k] for k in CONFIG_KEYS})
        layers = (LlamaLayer * cfg["n_layers"])()
        for i, L in enumerate(weights["layers"]):
            layers[i].input_norm = P(L["input_norm"].data_ptr())
            layers[i].post_norm = P(L["post_norm"].data_ptr())
            for n in PROJ:
                setattr(layers[i], n, _qw(L[n]))
        embed = _qw(weights["embed"])
        head = _qw(weights.get("lm_head"))
        self.handle = P()
        check(lib().nq_llama_create(ctypes.byref(self.handle), ctypes.byref(c), layers,
                                    P(weights["final_norm"].data_ptr()), ctypes.byref(embed),
                                    ctypes.byref(head) if head.w else None))
        self.vocab = cfg["vocab"]

    def close(self):
        if self.handle:
            lib().nq_llama_destroy(self.handle)
            self.handle = P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def position(self):
        return int(lib().nq_llama_position(self.handle))

    def reset(self):
        check(lib().nq_llama_reset(self.handle, ops._stream()))

    def step(self, token=None, logits=True):
        """One step on `token` (int32 CUDA tensor of 1; None: the last argmax).
        Returns (logits fp32 [vocab] or None, next token int32 [1])."""
        lg = torch.empty(self.vocab, dtype=torch.float32, device="cuda") if logits else None
        nxt = torch.empty(1, dtype=torch.int32, device="cuda")
        check(lib().nq_llama_step(self.handle, P(token.data_ptr()) if token is not None else None,
                                  P(lg.data_ptr()) if lg is not None else None,
                                  P(nxt.data_ptr()), ops._stream()))
        return lg, nxt

    def prefill(self, tokens, logits=True):
        """The prompt (int32 CUDA tensor) through the decoder, one position per
        step; returns the last position's logits (fp32) or None."""
        if tokens.dtype != torch.int32 or not tokens.is_cuda:
            raise NQError(1, "prefill: tokens must be an int32 CUDA tensor")
        lg = torch.empty(self.vocab, dtype=torch.float32, device="cuda") if logits else None
        check(lib().nq_llama_prefill(self.handle, P(tokens.data_ptr()), tokens.numel(),
                                     P(lg.data_ptr()) if lg is not None else None,
                                     ops._stream()))
        return lg

    def generate(self, n, token=None, out=None):
        """n greedy steps, pipelined on the device; returns the n tokens."""
        out = out if out is not None else torch.empty(n, dtype=torch.int32, device="cuda")
        check(lib().nq_llama_generate(self.handle,
                                      P(token.data_ptr()) if token is not None else None, n,
                                      P(out.data_ptr()), ops._stream()))
        return out
