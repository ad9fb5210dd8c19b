"""fp16 checkpoints: scales and biases stored as fp16 (mlx_ops::lin,
compute/src/compute/model/mlx_ops.h:33-39, passes whatever dtype the
checkpoint holds; the activations then run in fp16).  Quantize and dequantize
are bit-exact against the oracle's fp16 restatement (dequant =
fp16(fp16(s*q) + b)); the fp16 quantized matmul, on both kernels (the decode
GEMV for M <= 8, the tcgen05 GEMM otherwise), meets the matmul tolerance.
(cuda_ops::lin over a checkpoint with F16 scales: tests/test_cpp_backend.py.)"""
import numpy as np
import pytest
import torch

from _util import MAX_REL, MEAN_REL, dev_u32, host_u16, host_u32, rel_errors, weights

pytestmark = pytest.mark.gpu


def dev_f16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.float16)).cuda()


def f16_bits(a):
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def assert_close_f16(y_bits, ref_bits, what):
    y = y_bits.view(np.float16).astype(np.float64)
    r = ref_bits.view(np.float16).astype(np.float64)
    rel = rel_errors(y, r)
    assert np.isfinite(y).all(), what
    assert rel.max() <= MAX_REL and rel.mean() <= MEAN_REL, (what, rel.max(), rel.mean())


@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (8, 64), (8, 128)])
@pytest.mark.parametrize("scheme", [0, 1])
def test_quantize_f16_bit_exact(oracle, nqlib, bits, gs, scheme):
    import neurons_b200 as nb
    rng = np.random.default_rng(bits * 10 + gs + scheme)
    w = weights(rng, 29, 512)
    w[0, :gs] = 0.25
    w[1, :gs] = 0.0
    wb = f16_bits(w)
    ref = oracle.quantize(wb, bits, gs, scheme, f16=True)
    got = nb.quantize(dev_f16(wb), gs, bits, scheme)
    assert got[1].dtype == torch.float16
    np.testing.assert_array_equal(host_u32(got[0]), ref[0])
    np.testing.assert_array_equal(host_u16(got[1]), ref[1])
    np.testing.assert_array_equal(host_u16(got[2]), ref[2])


@pytest.mark.parametrize("bits,gs", [(4, 64), (4, 128), (8, 32), (8, 64)])
def test_dequantize_f16_bit_exact(oracle, nqlib, bits, gs):
    """Random codes and fp16 scales/biases over a wide exponent range
    (subnormal products included)."""
    import neurons_b200 as nb
    rng = np.random.default_rng(bits + 3 * gs)
    wq = rng.integers(0, 2 ** 32, size=(48, 256), dtype=np.uint64).astype(np.uint32)
    K = 256 * 32 // bits
    s = f16_bits(rng.standard_normal((48, K // gs)) * 10.0 ** rng.uniform(-7, 1, (48, K // gs)))
    b = f16_bits(rng.standard_normal((48, K // gs)) * 10.0 ** rng.uniform(-7, 1, (48, K // gs)))
    ref = oracle.dequantize(wq, s, b, bits, gs, f16=True)
    got = nb.dequantize(dev_u32(wq), dev_f16(s), dev_f16(b), gs, bits)
    assert got.dtype == torch.float16
    np.testing.assert_array_equal(host_u16(got), ref)


@pytest.mark.parametrize("M", [1, 3, 8, 9, 33, 300])
@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_f16(oracle, nqlib, M, bits):
    import neurons_b200 as nb
    rng = np.random.default_rng(M * 5 + bits)
    N, K, gs = 256, 2048, 64
    wq, s, b = oracle.quantize(f16_bits(weights(rng, N, K)), bits, gs, 0, f16=True)
    x = f16_bits(rng.standard_normal((M, K)))
    y = nb.quantized_matmul(dev_f16(x), dev_u32(wq), dev_f16(s), dev_f16(b), True, gs, bits)
    torch.cuda.synchronize()
    assert y.dtype == torch.float16 and nb.take_device_error() == 0
    assert_close_f16(host_u16(y), oracle.qmm(x, wq, s, b, bits, gs, f16=True),
                     f"fp16 qmm M={M} bits={bits}")


def test_qmm_f16_prefill_shape(oracle, nqlib):
    """M=2048 x [14336, 4096] on the tensor cores, sampled weight rows checked."""
    import neurons_b200 as nb
    g = torch.Generator(device="cuda").manual_seed(5)
    M, N, K = 2048, 14336, 4096
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    wq, s, b = nb.quantize(w, 64, 4)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    y = nb.quantized_matmul(x, wq, s, b, True, 64, 4)
    torch.cuda.synchronize()
    rows = np.random.default_rng(1).choice(N, 64, replace=False)
    ref = oracle.qmm(host_u16(x), host_u32(wq)[rows], host_u16(s)[rows], host_u16(b)[rows], 4,
                     64, f16=True)
    assert_close_f16(host_u16(y)[:, rows], ref, "fp16 prefill")
