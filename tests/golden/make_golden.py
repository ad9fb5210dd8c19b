"""Generate the golden fixtures under tests/golden/ (committed).

    python tests/golden/make_golden.py

Inputs are seeded synthetic tensors (numpy PCG64) with the workload's value
distributions (weights N(0, 0.02), activations N(0, 1) rounded to bf16,
router logits N(0, 1)); expected outputs come from the C oracle
(oracle/nq_oracle.c) and are cross-checked here against the independent numpy
restatement (oracle/np_oracle.py) before being written.  Known-answer cases
with hand-derived codes are written alongside.

The reference (neurons) ships no quantized-matmul fixture that can be used
without the TinyLlama checkpoint, and MLX itself cannot run here, so these
fixtures pin the restatement, not MLX.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import np_oracle as N  # noqa: E402
from oracle import oracle as O  # noqa: E402


def bf16(a):
    return O.f32_to_bf16(np.asarray(a, np.float32))


def known_answers():
    """Hand-derived cases (codes written out by reasoning, not by the oracle)."""
    cases = {}
    # 1. a group whose values are exactly 0..15 times 0.5 under the minmax scheme:
    #    scale = 7.5/15 = 0.5, bias = 0, codes = 0..15, packed little-nibble-first.
    w = np.tile(np.arange(32, dtype=np.float32) % 16 * 0.5, (2, 1))
    cases["ka_ramp_w"] = w
    cases["ka_ramp_wq"] = np.array([[0x76543210, 0xFEDCBA98, 0x76543210, 0xFEDCBA98]] * 2,
                                   np.uint32)
    cases["ka_ramp_scales"] = bf16([[0.5], [0.5]])
    cases["ka_ramp_biases"] = bf16([[0.0], [0.0]])
    # 2. a constant group (max == min): minmax scale 0 -> all codes 0, bias = value.
    cases["ka_const_w"] = np.full((1, 32), 0.25, np.float32)
    cases["ka_const_wq"] = np.zeros((1, 4), np.uint32)
    cases["ka_const_scales"] = bf16([[0.0]])
    cases["ka_const_biases"] = bf16([[0.25]])
    # 3. MLX scheme on a ramp 0..15 (|max| > |min|): scale = -(15/15) = -1,
    #    edge = max = 15, q0 = rint(15 / -1) = -15, scale = 15 / -15 = -1,
    #    bias = 15, codes = rint((w - 15) / -1) = 15 - w.
    w3 = np.tile(np.arange(16, dtype=np.float32), (1, 2))
    cases["ka_mlx_w"] = w3
    cases["ka_mlx_wq"] = np.array([[0x89ABCDEF, 0x01234567, 0x89ABCDEF, 0x01234567]], np.uint32)
    cases["ka_mlx_scales"] = bf16([[-1.0]])
    cases["ka_mlx_biases"] = bf16([[15.0]])
    # 4. 8-bit packing (minmax, two groups of 128 over the values 0..255): per group
    #    max - min = 127, scale = 127/255, codes = rint((w - min) / scale) span 0..255,
    #    four codes per word, lowest index in the lowest byte.
    w4 = np.arange(256, dtype=np.float32)[None, :]
    cases["ka_8bit_w"] = w4
    sc = np.float32(np.float32(127) / np.float32(255))
    g0 = np.rint(np.arange(128, dtype=np.float32) / sc)
    g1 = np.rint((np.arange(128, 256, dtype=np.float32) - np.float32(128)) / sc)
    q4 = np.concatenate([g0, g1]).astype(np.uint32).reshape(1, 64, 4)
    cases["ka_8bit_wq"] = (q4[..., 0] | (q4[..., 1] << 8) | (q4[..., 2] << 16) |
                           (q4[..., 3] << 24)).astype(np.uint32)
    # 5. dequantize rounds twice, like MLX's bf16 arithmetic: bf16(bf16(s*q) + b).
    #    s = bf16 0x3B09 = 2^-9 * (1 + 9/128) = 0.0020904541015625, q = 14, b = 0.75.
    #    s*q = 0.029266357421875 = 2^-6 * 239.75/128 -> bf16 2^-6 * 240/128 = 0.029296875;
    #    + 0.75 = 0.779296875 = 199.5 * 2^-8 -> tie -> even 200 * 2^-8 = 0.78125 = 0x3F48.
    #    (A single rounding of the exact s*q + b = 199.49 * 2^-8 would give 0x3F47.)
    cases["ka_dq_wq"] = np.full((1, 4), 0xEEEEEEEE, np.uint32)  # 32 codes, all 14
    cases["ka_dq_scales"] = np.array([[0x3B09]], np.uint16)
    cases["ka_dq_biases"] = bf16([[0.75]])
    cases["ka_dq_out"] = np.full((1, 32), 0x3F48, np.uint16)
    return cases


def seeded_cases():
    rng = np.random.default_rng(0)
    out = {}
    for bits in (4, 8):
        for gs in (32, 64, 128):
            for scheme in (0, 1):
                tag = f"b{bits}_g{gs}_s{scheme}"
                w = (rng.standard_normal((40, 256)) * 0.02).astype(np.float32)
                wq, s, b = O.quantize(w, bits, gs, scheme)
                nq, ns, nb = N.quantize(w, bits, gs, scheme)
                assert (wq == nq).all() and (s == ns).all() and (b == nb).all(), tag
                dq = O.dequantize(wq, s, b, bits, gs)
                assert (dq == N.dequantize(wq, s, b, bits, gs)).all(), tag
                x = bf16(rng.standard_normal((5, 256)))
                y, y32 = O.qmm(x, wq, s, b, bits, gs, want_f32=True)
                ref = N.qmm_f64(x, wq, s, b, bits, gs)
                assert np.abs(y32 - ref).max() < 1e-5, tag
                out.update({f"{tag}_w": w, f"{tag}_wq": wq, f"{tag}_s": s, f"{tag}_b": b,
                            f"{tag}_dq": dq, f"{tag}_x": x, f"{tag}_y": y})
    # MoE routing + switch step at small dims (E=16, k=4, H=64, I=32)
    T, E, k, H, I = 6, 16, 4, 64, 32
    logits = bf16(rng.standard_normal((T, E)))
    idx, sc = O.moe_route(logits, k)
    x = bf16(rng.standard_normal((T, H)))
    mats = {}
    for name, rows, cols in (("gate", I, H), ("up", I, H), ("down", H, I)):
        w = (rng.standard_normal((E * rows, cols)) * 0.02).astype(np.float32)
        wq, s, b = O.quantize(w, 4, 32, 0)
        mats[name] = (wq.reshape(E, rows, -1), s.reshape(E, rows, -1), b.reshape(E, rows, -1))
    y_fused = O.moe_switch(x, idx, sc, mats["gate"], mats["up"], mats["down"], 4, 32, rounding=1)
    y_mlx = O.moe_switch(x, idx, sc, mats["gate"], mats["up"], mats["down"], 4, 32, rounding=0)
    out.update({"moe_logits": logits, "moe_idx": idx, "moe_scores": sc, "moe_x": x,
                "moe_y_fused": y_fused, "moe_y_mlx": y_mlx})
    for name in ("gate", "up", "down"):
        out[f"moe_{name}_wq"], out[f"moe_{name}_s"], out[f"moe_{name}_b"] = mats[name]
    # gather_qmm, decode shape family (x [1, K] broadcast over 3 indices)
    gx = bf16(rng.standard_normal((1, 1, 64)))
    rhs = np.array([5, 0, 15], np.int32)
    gout = O.gather_qmm(gx, mats["gate"][0], mats["gate"][1], mats["gate"][2], rhs,
                        bits=4, group_size=32)
    out.update({"gq_x": gx, "gq_rhs": rhs, "gq_out": gout})
    return out


def main():
    ka = known_answers()
    np.savez_compressed(os.path.join(HERE, "known_answers.npz"), **ka)
    sc = seeded_cases()
    np.savez_compressed(os.path.join(HERE, "seeded_small.npz"), **sc)
    print("wrote", len(ka), "known-answer arrays and", len(sc), "seeded arrays")


if __name__ == "__main__":
    main()
