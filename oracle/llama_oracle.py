"""CPU restatement of the reference's Llama decode step -- test infrastructure.

Only tests/ (and bench.py's CPU-baseline legs) use this module; nothing in
neurons_b200/ imports it.  It follows the compiled decode function of
compute/src/compute/model/llama_model.cpp:355-509 op by op, with MLX's bf16
rounding after every op (each op computed in fp32 and rounded to bf16):

  h = embed[token]                              dequantized row (:384, :60-72)
  x = rms_norm(h, input_layernorm, eps)          (:392)
  q, k, v = lin(x, q/k/v_proj)                   (:394-396; mlx_ops.h:28-42)
  q, k = rope(q, pos), rope(k, pos)              (:446-455; traditional=false)
  K, V = concat(K, k), concat(V, v)              (:458-461)
  a = sdpa(q, K, V, scale=1/sqrt(head_dim))      (:463-470; GQA)
  h = h + lin(a, o_proj)                         (:476)
  x = rms_norm(h, post_attention_layernorm)      (:478-479)
  h = h + lin(sigmoid(g) * g * u, down_proj), g, u = lin(x, gate/up_proj)
                                                 (:480-483)
  logits = lin(rms_norm(h, norm), lm_head) or matmul(h, embed^T)  (:486-495)
  next = argmax(logits)                          (:745-790, greedy)

Decisions MLX leaves open here (its kernels are not in the reference tree):
rms_norm = bf16(w * bf16(x * 1/sqrt(mean(x^2) + eps))) with the sum of
squares in fp32; rope angle = pos * 2^(-(i / (d/2)) * log2(theta)) in fp32,
rotation in fp32, rounded to bf16; attention scores in fp64 over the bf16
q and cached k, softmax and the weighted sum of bf16 v in fp64, output
rounded to bf16.  The tied LM head is the 4-bit qmm over the quantized
embedding, which equals matmul(h, dequantize(embed)^T) up to summation order.
"""
import numpy as np

from . import oracle as O


def bf16(a):
    """Round fp32/fp64 values to bf16, returned as fp32 values."""
    return O.bf16_to_f32(O.f32_to_bf16(np.asarray(a, np.float32)))


def rms_norm(x, w, eps):
    x = np.asarray(x, np.float32)
    ss = np.sum(x * x, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(np.float32(ss / np.float32(x.size)) + np.float32(eps))
    return bf16(np.asarray(w, np.float32) * bf16(x * inv))


def rope(x, pos, theta):
    """x [heads, d] (bf16 values as fp32) rotated at position pos."""
    d = x.shape[-1]
    half = d // 2
    i = np.arange(half, dtype=np.float32)
    inv_freq = np.exp2(-(i / np.float32(half)) * np.float32(np.log2(np.float32(theta))))
    ang = (np.float32(pos) * inv_freq).astype(np.float64)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    x1, x2 = x[..., :half], x[..., half:]
    return bf16(np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1))


def lin(x, wq, s, b, bits, gs):
    return O.bf16_to_f32(O.qmm(O.f32_to_bf16(np.asarray(x, np.float32)[None]), wq, s, b,
                               bits, gs))[0]


class LlamaOracle:
    """weights: dict with 'embed' (wq, s, b), 'final_norm', optional 'lm_head'
    (wq, s, b), and 'layers': list of dicts with 'input_norm', 'post_norm' (bf16
    bit patterns) and 'q','k','v','o','gate','up','down' (wq, s, b)."""

    def __init__(self, cfg, weights):
        self.c = cfg
        self.w = weights
        self.K = [[] for _ in weights["layers"]]
        self.V = [[] for _ in weights["layers"]]
        self.pos = 0

    def step(self, token):
        c, W = self.c, self.w
        bits, gs = c["bits"], c["group_size"]
        H, nh, nkv, hd = c["hidden"], c["n_heads"], c["n_kv_heads"], c["head_dim"]
        ew, es, eb = W["embed"]
        h = O.bf16_to_f32(O.dequantize(ew[token:token + 1], es[token:token + 1],
                                       eb[token:token + 1], bits, gs))[0]
        f = lambda a: O.bf16_to_f32(a)
        for li, L in enumerate(W["layers"]):
            x = rms_norm(h, f(L["input_norm"]), c["rms_eps"])
            q = lin(x, *L["q"], bits, gs).reshape(nh, hd)
            k = lin(x, *L["k"], bits, gs).reshape(nkv, hd)
            v = lin(x, *L["v"], bits, gs).reshape(nkv, hd)
            q = rope(q, self.pos, c["rope_theta"])
            k = rope(k, self.pos, c["rope_theta"])
            self.K[li].append(k)
            self.V[li].append(v)
            Kc = np.stack(self.K[li], axis=1).astype(np.float64)  # [nkv, T, hd]
            Vc = np.stack(self.V[li], axis=1).astype(np.float64)
            g = nh // nkv
            a = np.zeros((nh, hd), np.float64)
            for hh in range(nh):
                j = hh // g
                sc = (Kc[j] @ q[hh].astype(np.float64)) / np.sqrt(hd)
                p = np.exp(sc - sc.max())
                a[hh] = (p / p.sum()) @ Vc[j]
            a = bf16(a.reshape(-1))
            h = bf16(h + lin(a, *L["o"], bits, gs))
            x = rms_norm(h, f(L["post_norm"]), c["rms_eps"])
            gt = lin(x, *L["gate"], bits, gs)
            up = lin(x, *L["up"], bits, gs)
            sg = bf16(1.0 / (1.0 + np.exp(-gt.astype(np.float32))))
            m = bf16(bf16(sg * gt) * up)
            h = bf16(h + lin(m, *L["down"], bits, gs))
        x = rms_norm(h, f(W["final_norm"]), c["rms_eps"])
        head = W.get("lm_head") or W["embed"]
        logits = lin(x, *head, bits, gs)
        self.pos += 1
        return logits, int(np.argmax(logits))
