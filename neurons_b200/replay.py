"""Decode-step replay of LlamaModel's quantized linears.

LlamaModel's decode function (compute/src/compute/model/llama_model.cpp:393-494)
makes, per decoder layer, seven `lin()` calls in this order:

    q_proj, k_proj, v_proj   on rms_norm(h)                         (:400-402)
    o_proj                   on the attention output                (:480)
    gate_proj, up_proj       on rms_norm(h + o)                     (:484-485)
    down_proj                on silu(gate) * up                     (:486-487)

and one `lin(h, "lm_head")` after the last layer (:492-494).  The model is
written against mx::array and its norm, RoPE, attention and SwiGLU ops are
MLX's, outside the quantized-matmul path, so this harness replays only the
`lin()` sequence: the same weight names, shapes, order and data dependencies,
with each non-linear step replaced by passing the producing projection's
output on (o_proj reads q_proj's output, gate/up read o_proj's output,
down_proj reads gate_proj's output, the next layer reads down_proj's output).
Every call goes through `ops.lin`, i.e. through the C ABI.
"""
import torch

from . import ops


class LlamaDecodeReplay:
    """Quantized weights of a Llama-shaped model in MLX's layout, keyed like the
    checkpoint ("model.layers.{i}.self_attn.q_proj.weight" / ".scales" /
    ".biases"), and the device buffers of one decode step."""

    def __init__(self, hidden=3072, n_heads=24, n_kv=8, head_dim=128, inter=8192, layers=28,
                 vocab=128256, bits=4, group_size=64, seed=0, device="cuda",
                 scheme=ops.SCHEME_MINMAX):
        self.hidden, self.inter, self.layers, self.vocab = hidden, inter, layers, vocab
        self.q_dim, self.kv_dim = n_heads * head_dim, n_kv * head_dim
        self.bits, self.gs = bits, group_size
        self.wm = {}
        g = torch.Generator(device=device).manual_seed(seed)
        for i in range(layers):
            a = f"model.layers.{i}.self_attn."
            m = f"model.layers.{i}.mlp."
            for key, n, k in ((a + "q_proj", self.q_dim, hidden), (a + "k_proj", self.kv_dim, hidden),
                              (a + "v_proj", self.kv_dim, hidden), (a + "o_proj", hidden, self.q_dim),
                              (m + "gate_proj", inter, hidden), (m + "up_proj", inter, hidden),
                              (m + "down_proj", hidden, inter)):
                self._add(key, n, k, g, device, scheme)
        self._add("lm_head", vocab, hidden, g, device, scheme)
        bf = dict(dtype=torch.bfloat16, device=device)
        self.x = torch.empty(1, hidden, **bf)
        self.q = torch.empty(1, self.q_dim, **bf)
        self.k = torch.empty(1, self.kv_dim, **bf)
        self.v = torch.empty(1, self.kv_dim, **bf)
        self.o = torch.empty(1, hidden, **bf)
        self.gate = torch.empty(1, inter, **bf)
        self.up = torch.empty(1, inter, **bf)
        self.h = torch.empty(1, hidden, **bf)
        self.logits = torch.empty(1, vocab, **bf)

    def _add(self, key, n, k, g, device, scheme):
        w = torch.randn(n, k, device=device, generator=g) * 0.02
        wq, s, b = ops.quantize(w, self.gs, self.bits, scheme)
        del w
        self.wm[key + ".weight"], self.wm[key + ".scales"], self.wm[key + ".biases"] = wq, s, b

    def weight_bytes(self):
        """Bytes of packed codes, scales and biases one token reads."""
        return sum(t.numel() * t.element_size() for t in self.wm.values())

    def algorithmic_bytes(self):
        """Weights plus each call's activation read and output write."""
        act = 0
        for key, w in self.wm.items():
            if key.endswith(".weight"):
                n, k = int(w.shape[0]), int(w.shape[1]) * 32 // self.bits
                act += 2 * (n + k)
        return self.weight_bytes() + act

    def launches_per_token(self):
        return 7 * self.layers + 1

    def step(self):
        """One decode token: reads self.x, leaves the logits in self.logits."""
        wm, gs = self.wm, self.gs
        h = self.x
        for i in range(self.layers):
            a = f"model.layers.{i}.self_attn."
            m = f"model.layers.{i}.mlp."
            ops.lin(h, a + "q_proj", wm, gs, out=self.q)
            ops.lin(h, a + "k_proj", wm, gs, out=self.k)
            ops.lin(h, a + "v_proj", wm, gs, out=self.v)
            ops.lin(self.q, a + "o_proj", wm, gs, out=self.o)
            ops.lin(self.o, m + "gate_proj", wm, gs, out=self.gate)
            ops.lin(self.o, m + "up_proj", wm, gs, out=self.up)
            ops.lin(self.gate, m + "down_proj", wm, gs, out=self.h)
            h = self.h
        ops.lin(h, "lm_head", wm, gs, out=self.logits)
        return self.logits
