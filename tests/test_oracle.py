"""CPU tests of the oracle: known answers, committed golden fixtures, and the
C restatement against the independent numpy restatement."""
import os

import numpy as np
import pytest

from oracle import np_oracle as N

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ka():
    return np.load(os.path.join(GOLDEN, "known_answers.npz"))


@pytest.fixture(scope="module")
def seeded():
    return np.load(os.path.join(GOLDEN, "seeded_small.npz"))


@pytest.mark.parametrize("case,scheme,bits,gs", [
    ("ramp", 1, 4, 32), ("const", 1, 4, 32), ("mlx", 0, 4, 32), ("8bit", 1, 8, 128)])
def test_known_answers_quantize(oracle, ka, case, scheme, bits, gs):
    wq, s, b = oracle.quantize(ka[f"ka_{case}_w"], bits, gs, scheme)
    np.testing.assert_array_equal(wq, ka[f"ka_{case}_wq"])
    if f"ka_{case}_scales" in ka:
        np.testing.assert_array_equal(s, ka[f"ka_{case}_scales"])
        np.testing.assert_array_equal(b, ka[f"ka_{case}_biases"])


def test_known_answer_dequant_double_rounding(oracle, ka):
    out = oracle.dequantize(ka["ka_dq_wq"], ka["ka_dq_scales"], ka["ka_dq_biases"], 4, 32)
    np.testing.assert_array_equal(out, ka["ka_dq_out"])


def test_known_answer_packing_order(oracle):
    # code j of a word sits in bits [bits*j, bits*(j+1)): a word 0x76543210 with
    # scale 1 and bias 0 dequantizes to 0, 1, ..., 7
    wq = np.array([[0x76543210, 0xFEDCBA98, 0, 0]], np.uint32)
    one = oracle.f32_to_bf16(np.array([[1.0]], np.float32))
    zero = oracle.f32_to_bf16(np.array([[0.0]], np.float32))
    out = oracle.bf16_to_f32(oracle.dequantize(wq, one, zero, 4, 32))
    np.testing.assert_array_equal(out[0, :16], np.arange(16, dtype=np.float32))


@pytest.mark.parametrize("w_cols,s_cols,gs,expect", [
    (512, 64, 64, 4), (1024, 64, 64, 8), (256, 32, 64, 4), (96, 12, 64, 4), (192, 12, 64, 8),
    (0, 64, 64, 4), (512, 128, 32, 4), (1024, 32, 128, 8)])
def test_bits_from_shapes(oracle, w_cols, s_cols, gs, expect):
    # mlx_ops.h:20-25
    assert oracle.bits_from_shapes(w_cols, s_cols, gs) == expect


def test_golden_seeded_reproduces(oracle, seeded):
    for bits in (4, 8):
        for gs in (32, 64, 128):
            for scheme in (0, 1):
                tag = f"b{bits}_g{gs}_s{scheme}"
                wq, s, b = oracle.quantize(seeded[f"{tag}_w"], bits, gs, scheme)
                np.testing.assert_array_equal(wq, seeded[f"{tag}_wq"])
                np.testing.assert_array_equal(s, seeded[f"{tag}_s"])
                np.testing.assert_array_equal(b, seeded[f"{tag}_b"])
                np.testing.assert_array_equal(oracle.dequantize(wq, s, b, bits, gs),
                                              seeded[f"{tag}_dq"])
                np.testing.assert_array_equal(
                    oracle.qmm(seeded[f"{tag}_x"], wq, s, b, bits, gs), seeded[f"{tag}_y"])


def test_golden_moe_reproduces(oracle, seeded):
    idx, sc = oracle.moe_route(seeded["moe_logits"], 4)
    np.testing.assert_array_equal(idx, seeded["moe_idx"])
    np.testing.assert_array_equal(sc, seeded["moe_scores"])
    mats = {n: (seeded[f"moe_{n}_wq"], seeded[f"moe_{n}_s"], seeded[f"moe_{n}_b"])
            for n in ("gate", "up", "down")}
    y = oracle.moe_switch(seeded["moe_x"], idx, sc, mats["gate"], mats["up"], mats["down"],
                          4, 32, rounding=1)
    np.testing.assert_array_equal(y, seeded["moe_y_fused"])
    # the fused rounding points and MLX's op chain agree to bf16 precision
    a = oracle.bf16_to_f32(seeded["moe_y_fused"]).astype(np.float64)
    b = oracle.bf16_to_f32(seeded["moe_y_mlx"]).astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 2e-2


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("scheme", [0, 1])
@pytest.mark.parametrize("in_bf16", [False, True])
def test_c_vs_numpy_restatement(oracle, bits, gs, scheme, in_bf16):
    rng = np.random.default_rng(bits * 1000 + gs * 10 + scheme)
    w = (rng.standard_normal((33, 384)) * 0.02).astype(np.float32)
    # edges: a constant group, an all-zero group, large magnitudes
    w[0, :gs] = 0.125
    w[1, :gs] = 0.0
    w[2, :gs] *= 1000
    if in_bf16:
        w = oracle.f32_to_bf16(w)
    a = oracle.quantize(w, bits, gs, scheme)
    b = N.quantize(w, bits, gs, scheme)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)
    np.testing.assert_array_equal(oracle.dequantize(*a, bits, gs), N.dequantize(*a, bits, gs))


@pytest.mark.parametrize("scheme,bound", [(1, 0.5), (0, 1.25)])
def test_dequant_error_bound(oracle, scheme, bound):
    """Round-trip error per element is within bound * |scale| plus the bf16
    roundings of scale, bias and result.  The MLX scheme snaps one group edge
    onto the grid, which can push the far edge one code past the range
    (clamped), hence its looser bound."""
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((64, 512)) * 0.02).astype(np.float32)
    wq, s, b = oracle.quantize(w, 4, 64, scheme)
    wh = oracle.bf16_to_f32(oracle.dequantize(wq, s, b, 4, 64))
    sc = np.abs(np.repeat(oracle.bf16_to_f32(s), 64, axis=1))
    bb = np.abs(np.repeat(oracle.bf16_to_f32(b), 64, axis=1))
    slack = 15 * sc * 2 ** -8 + bb * 2 ** -8 + np.abs(w) * 2 ** -8
    assert (np.abs(w - wh) <= bound * sc + slack).all()


def test_qmm_against_numpy_f64(oracle):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((17, 256)) * 0.02).astype(np.float32)
    x = oracle.f32_to_bf16(rng.standard_normal((7, 256)).astype(np.float32))
    wq, s, b = oracle.quantize(w, 4, 64, 0)
    _, y32 = oracle.qmm(x, wq, s, b, 4, 64, want_f32=True)
    ref = N.qmm_f64(x, wq, s, b, 4, 64)
    np.testing.assert_allclose(y32, ref, rtol=1e-6, atol=1e-6)


def test_gather_qmm_semantics(oracle, seeded):
    x = seeded["gq_x"]
    out = oracle.gather_qmm(x, seeded["moe_gate_wq"], seeded["moe_gate_s"], seeded["moe_gate_b"],
                            seeded["gq_rhs"], bits=4, group_size=32)
    np.testing.assert_array_equal(out, seeded["gq_out"])
    # each slice equals a plain qmm against the selected expert
    for i, e in enumerate(seeded["gq_rhs"]):
        y = oracle.qmm(x[0], seeded["moe_gate_wq"][e], seeded["moe_gate_s"][e],
                       seeded["moe_gate_b"][e], 4, 32)
        np.testing.assert_array_equal(out[i], y)


def test_oracle_rejects_bad_shapes(oracle):
    with pytest.raises(ValueError):
        oracle.quantize(np.zeros((4, 48), np.float32), 4, 32)      # K % gs != 0
    with pytest.raises(ValueError):
        oracle.quantize(np.zeros((4, 64), np.float32), 3, 32)      # unsupported bits


def test_route_ties_prefer_lower_index(oracle):
    logits = oracle.f32_to_bf16(np.array([[0.5, 1.0, 1.0, 0.25, 1.0]], np.float32))
    idx, sc = oracle.moe_route(logits, 2)
    np.testing.assert_array_equal(idx, [[1, 2]])
    np.testing.assert_allclose(sc, [[0.5, 0.5]], rtol=1e-7)


def test_f16_conversion_matches_ieee_rne(oracle):
    """The oracle's fp32 -> fp16 conversion (fp16 checkpoints) is IEEE
    round-to-nearest-even, checked against numpy's float16 over normal,
    subnormal, overflow and tie cases."""
    rng = np.random.default_rng(5)
    v = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    edges = np.array([65504, 65519, 65520, 65536, 1e-8, 6e-8, 2.98e-8, 6.1e-5, 6.09e-5,
                      1 + 2 ** -11, 1 + 3 * 2 ** -11, -0.0, 0.0, np.inf, -np.inf], np.float32)
    v = np.concatenate([v, edges])
    with np.errstate(over="ignore"):
        ref = v.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(oracle.f32_to_f16(v), ref)


def test_f16_dequant_and_qmm_follow_the_definition(oracle):
    """fp16 dequant = fp16(fp16(s*q) + b) (numpy float16 ops round the same
    way), and the fp16 qmm equals an fp64 dot over those values."""
    rng = np.random.default_rng(6)
    w = (rng.standard_normal((16, 256)) * 0.05).astype(np.float16)
    wq, s, b = oracle.quantize(w.view(np.uint16), 4, 64, 0, f16=True)
    dq = oracle.dequantize(wq, s, b, 4, 64, f16=True).view(np.float16)
    codes = np.stack([(wq >> (4 * i)) & 15 for i in range(8)], axis=-1).reshape(16, 256)
    sf = np.repeat(s.view(np.float16).astype(np.float32), 64, axis=1)
    bf = np.repeat(b.view(np.float16).astype(np.float32), 64, axis=1)
    ref = ((sf * codes).astype(np.float16).astype(np.float32) + bf).astype(np.float16)
    np.testing.assert_array_equal(dq.view(np.uint16), ref.view(np.uint16))
    x = rng.standard_normal((3, 256)).astype(np.float16)
    y = oracle.qmm(x.view(np.uint16), wq, s, b, 4, 64, f16=True).view(np.float16)
    yr = (x.astype(np.float64) @ dq.astype(np.float64).T).astype(np.float32).astype(np.float16)
    np.testing.assert_array_equal(y, yr)
