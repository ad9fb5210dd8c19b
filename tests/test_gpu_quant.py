"""GPU parity: quantize/pack and dequantize through the C ABI are bit-exact
against the oracle (codes, scales, biases, dequantized bf16)."""
import os

import numpy as np
import pytest

from _util import dev_bf16, dev_f32, dev_u32, host_u16, host_u32, weights

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("scheme", [0, 1])
@pytest.mark.parametrize("in_bf16", [False, True])
def test_quantize_bit_exact(oracle, nqlib, bits, gs, scheme, in_bf16):
    import neurons_b200 as nb
    rng = np.random.default_rng(bits * 7 + gs + scheme * 3 + in_bf16)
    w = weights(rng, 37, 640)
    w[0, :gs] = 0.125       # constant group
    w[1, :gs] = 0.0         # all-zero group
    w[2, :gs] *= 1000.0     # large magnitudes
    if in_bf16:
        w = oracle.f32_to_bf16(w)
        wd = dev_bf16(w)
    else:
        wd = dev_f32(w)
    ref = oracle.quantize(w, bits, gs, scheme)
    got = nb.quantize(wd, gs, bits, scheme)
    np.testing.assert_array_equal(host_u32(got[0]), ref[0])
    np.testing.assert_array_equal(host_u16(got[1]), ref[1])
    np.testing.assert_array_equal(host_u16(got[2]), ref[2])


@pytest.mark.parametrize("scheme", [0, 1])
def test_quantize_full_size_decode_shape(oracle, nqlib, scheme):
    """4096 x 4096 fp32 N(0, 0.02), 4-bit g64 (the decode workload's weight)."""
    import neurons_b200 as nb
    w = weights(np.random.default_rng(0), 4096, 4096)
    ref = oracle.quantize(w, 4, 64, scheme)
    got = nb.quantize(dev_f32(w), 64, 4, scheme)
    np.testing.assert_array_equal(host_u32(got[0]), ref[0])
    np.testing.assert_array_equal(host_u16(got[1]), ref[1])
    np.testing.assert_array_equal(host_u16(got[2]), ref[2])


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_dequantize_bit_exact(oracle, nqlib, bits, gs):
    import neurons_b200 as nb
    rng = np.random.default_rng(bits + gs)
    wq, s, b = oracle.quantize(weights(rng, 50, 1024), bits, gs, 0)
    ref = oracle.dequantize(wq, s, b, bits, gs)
    got = nb.dequantize(dev_u32(wq), dev_bf16(s), dev_bf16(b), gs, bits)
    np.testing.assert_array_equal(host_u16(got), ref)


def test_dequantize_random_scales_biases(oracle, nqlib):
    """Arbitrary bf16 scales/biases (negative scales, wide exponents) and random codes."""
    import neurons_b200 as nb
    rng = np.random.default_rng(11)
    wq = rng.integers(0, 2 ** 32, size=(64, 256), dtype=np.uint64).astype(np.uint32)
    s = oracle.f32_to_bf16((rng.standard_normal((64, 32)) * 10.0 ** rng.uniform(-6, 2, (64, 32)))
                           .astype(np.float32))
    b = oracle.f32_to_bf16((rng.standard_normal((64, 32)) * 10.0 ** rng.uniform(-6, 2, (64, 32)))
                           .astype(np.float32))
    for bits, gs in ((4, 64), (8, 64)):
        K = 256 * 32 // bits
        ss, bb = s[:, :K // gs], b[:, :K // gs]
        ref = oracle.dequantize(wq, ss, bb, bits, gs)
        got = nb.dequantize(dev_u32(wq), dev_bf16(ss), dev_bf16(bb), gs, bits)
        np.testing.assert_array_equal(host_u16(got), ref)


def test_dequantize_known_answer_double_rounding(nqlib):
    import neurons_b200 as nb
    ka = np.load(os.path.join(GOLDEN, "known_answers.npz"))
    got = nb.dequantize(dev_u32(ka["ka_dq_wq"]), dev_bf16(ka["ka_dq_scales"]),
                        dev_bf16(ka["ka_dq_biases"]), 32, 4)
    np.testing.assert_array_equal(host_u16(got), ka["ka_dq_out"])


def test_golden_seeded_quant(nqlib):
    import neurons_b200 as nb
    g = np.load(os.path.join(GOLDEN, "seeded_small.npz"))
    for bits in (4, 8):
        for gs in (32, 64, 128):
            for scheme in (0, 1):
                tag = f"b{bits}_g{gs}_s{scheme}"
                wq, s, b = nb.quantize(dev_f32(g[f"{tag}_w"]), gs, bits, scheme)
                np.testing.assert_array_equal(host_u32(wq), g[f"{tag}_wq"])
                np.testing.assert_array_equal(host_u16(s), g[f"{tag}_s"])
                np.testing.assert_array_equal(host_u16(b), g[f"{tag}_b"])
                np.testing.assert_array_equal(host_u16(nb.dequantize(wq, s, b, gs, bits)),
                                              g[f"{tag}_dq"])
