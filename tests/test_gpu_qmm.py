"""GPU parity: quantized_matmul through the C ABI against the oracle, on both
kernel paths (mma.sync GEMVs for a few tokens, TMA + tcgen05 GEMM otherwise;
the choice follows bits, M and the weight size), ragged
shapes, both bit widths and every group size, the golden fixtures, and the
full-size workloads (decode 4096x4096 at M=1; prefill 2048x14336x4096)."""
import os

import numpy as np
import pytest
import torch

from _util import (acts, assert_close, dev_bf16, dev_u32, host_u16, weights)

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def run_case(oracle, M, N, K, bits, gs, seed=0, scheme=0):
    import neurons_b200 as nb
    rng = np.random.default_rng(seed)
    wq, s, b = oracle.quantize(weights(rng, N, K), bits, gs, scheme)
    x = acts(rng, M, K)
    ref = oracle.qmm(x, wq, s, b, bits, gs)
    y = nb.quantized_matmul(dev_bf16(x), dev_u32(wq), dev_bf16(s), dev_bf16(b), True, gs, bits)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    return assert_close(host_u16(y), ref, f"M={M} N={N} K={K} bits={bits} gs={gs}")


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 16, 17, 24, 31, 32])
def test_gemv_path_m_sweep(oracle, nqlib, M):
    run_case(oracle, M, 80, 512, 4, 64, seed=M)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("M", [1, 7])
def test_gemv_path_bits_groups(oracle, nqlib, bits, gs, M):
    run_case(oracle, M, 48, 1024, bits, gs, seed=bits + gs)


@pytest.mark.parametrize("N,K", [(16, 32), (40, 96), (100, 160), (17, 4096), (1, 128),
                                 (3072, 3072), (1024, 3072), (3072, 8192)])
def test_gemv_path_ragged(oracle, nqlib, N, K):
    run_case(oracle, 1, N, K, 4, 32, seed=N)


@pytest.mark.parametrize("bits,gs,M,N,K", [(8, 32, 1, 100, 8192), (4, 64, 4, 48, 4096),
                                           (4, 128, 2, 33, 6144), (4, 32, 8, 24, 2048),
                                           (8, 64, 3, 40, 3072)])
def test_gemv_long_k_small_m(oracle, nqlib, bits, gs, M, N, K):
    """Decode shapes whose weight k-blocks outnumber the per-CTA ring (the ring
    wraps), scale spans that end inside a 64-group box, and up to 8 tokens."""
    run_case(oracle, M, N, K, bits, gs, seed=K + M)


@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (8, 32)])
def test_gemv_scales_at_any_bf16_alignment(oracle, nqlib, bits, gs):
    """Scales and biases handed over as views that start one bf16 element into
    their buffers (2-byte aligned, as a slice of a larger tensor can be): the
    result matches the oracle as with aligned buffers."""
    import neurons_b200 as nb
    rng = np.random.default_rng(bits * 7 + gs)
    M, N, K = 3, 64, 1024
    wq, s, b = oracle.quantize(weights(rng, N, K), bits, gs, 0)
    x = acts(rng, M, K)
    views = []
    for t in (s, b):
        buf = torch.empty(t.size + 1, dtype=torch.bfloat16, device="cuda")
        v = buf[1:].view(t.shape)
        v.copy_(dev_bf16(t))
        assert v.data_ptr() % 16 == 2
        views.append(v)
    y = nb.quantized_matmul(dev_bf16(x), dev_u32(wq), views[0], views[1], True, gs, bits)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    assert_close(host_u16(y), oracle.qmm(x, wq, s, b, bits, gs), f"offset scales b{bits} g{gs}")


def test_launch_count_query(nqlib):
    """The tail split is a second kernel only where a grid's last wave would run
    nearly empty (148 SMs): 2048 x 14336 has 896 = 6 x 148 + 8 tiles."""
    import neurons_b200 as nb
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert nb.quantized_matmul_launches(1, 4096, 4096) == 1          # GEMV
    tiles = (14336 // 128) * (2048 // 256)
    assert nb.quantized_matmul_launches(2048, 14336, 4096) == (2 if 0 < tiles % sms <= sms // 2
                                                               else 1)
    assert nb.quantized_matmul_launches(256, 4096, 4096) == 1        # all tiles split: tail only
    assert nb.quantized_matmul_launches(2048, 4096, 4096) in (1, 2)


@pytest.mark.parametrize("M", [33, 64, 65, 100, 128, 129, 200, 256, 257, 512])
def test_tc_path_m_sweep(oracle, nqlib, M):
    run_case(oracle, M, 256, 512, 4, 64, seed=M)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_tc_path_bits_groups(oracle, nqlib, bits, gs):
    run_case(oracle, 300, 384, 1024, bits, gs, seed=bits * gs)


@pytest.mark.parametrize("N,K", [(1, 64), (130, 96), (200, 160), (128, 4096), (257, 2048)])
def test_tc_path_ragged(oracle, nqlib, N, K):
    run_case(oracle, 96, N, K, 4, 32, seed=N + K)


@pytest.mark.parametrize("M,N,K", [(300, 512, 512), (2048, 1280, 1024), (200, 640, 2048)])
def test_tc_back_to_back_launches_are_ordered(oracle, nqlib, M, N, K):
    """y2 = W2 y1 right after y1 = W1 x on the stream: the second GEMM reads
    what the first one's tile stores (and split-tail clusters) wrote."""
    import neurons_b200 as nb
    rng = np.random.default_rng(M + N)
    w1 = oracle.quantize(weights(rng, N, K), 4, 64, 0)
    w2 = oracle.quantize(weights(rng, K, N), 4, 64, 0)
    x = acts(rng, M, K)
    d1 = [dev_u32(w1[0]), dev_bf16(w1[1]), dev_bf16(w1[2])]
    d2 = [dev_u32(w2[0]), dev_bf16(w2[1]), dev_bf16(w2[2])]
    xd = dev_bf16(x)
    for _ in range(3):
        y1 = nb.quantized_matmul(xd, *d1, True, 64, 4)
        y2 = nb.quantized_matmul(y1, *d2, True, 64, 4)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    assert_close(host_u16(y1), oracle.qmm(x, *w1, 4, 64), "tc chained stage 1")
    assert_close(host_u16(y2), oracle.qmm(host_u16(y1), *w2, 4, 64), "tc chained stage 2")


def test_golden_seeded_qmm(nqlib):
    import neurons_b200 as nb
    g = np.load(os.path.join(GOLDEN, "seeded_small.npz"))
    for bits in (4, 8):
        for gs in (32, 64, 128):
            for scheme in (0, 1):
                tag = f"b{bits}_g{gs}_s{scheme}"
                y = nb.quantized_matmul(dev_bf16(g[f"{tag}_x"]), dev_u32(g[f"{tag}_wq"]),
                                        dev_bf16(g[f"{tag}_s"]), dev_bf16(g[f"{tag}_b"]), True,
                                        gs, bits)
                assert_close(host_u16(y), g[f"{tag}_y"], tag)


def test_decode_config_full_size(oracle, nqlib):
    """M=1, N=K=4096, 4-bit g64, minmax scheme as the decode workload defines it."""
    run_case(oracle, 1, 4096, 4096, 4, 64, seed=0, scheme=1)


def test_prefill_config_full_size(oracle, nqlib):
    """M=2048, N=14336, K=4096, 4-bit g64: every output against a torch fp32 matmul
    of the bit-exact dequantized weights, plus 64 sampled weight rows against the
    oracle itself."""
    import neurons_b200 as nb
    M, N, K = 2048, 14336, 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.02
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    wq, s, b = nb.quantize(w, 64, 4, 1)
    y = nb.quantized_matmul(x, wq, s, b, True, 64, 4)
    wh = nb.dequantize(wq, s, b, 64, 4)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = x.float() @ wh.float().T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    assert_close(host_u16(y), oracle.f32_to_bf16(ref.cpu().numpy()), "prefill vs torch fp32")
    rows = np.random.default_rng(1).choice(N, 64, replace=False)
    wq_h = wq.cpu().view(torch.int32).numpy().view(np.uint32)[rows]
    s_h, b_h = host_u16(s)[rows], host_u16(b)[rows]
    ref_o = oracle.qmm(host_u16(x), wq_h, s_h, b_h, 4, 64)
    assert_close(host_u16(y)[:, rows], ref_o, "prefill vs oracle rows")
    np.testing.assert_array_equal(host_u16(wh)[rows], oracle.dequantize(wq_h, s_h, b_h, 4, 64))


def test_square_prefill_and_8bit(oracle, nqlib):
    """M=2048, N=K=4096 at 4 and 8 bits (sampled rows against the oracle)."""
    import neurons_b200 as nb
    M, N, K = 2048, 4096, 4096
    rng = np.random.default_rng(5)
    x = acts(rng, M, K)
    for bits in (4, 8):
        wq, s, b = oracle.quantize(weights(rng, N, K), bits, 64, 0)
        y = host_u16(nb.quantized_matmul(dev_bf16(x), dev_u32(wq), dev_bf16(s), dev_bf16(b),
                                          True, 64, bits))
        rows = rng.choice(N, 96, replace=False)
        ref = oracle.qmm(x, wq[rows], s[rows], b[rows], bits, 64)
        assert_close(y[:, rows], ref, f"square bits={bits}")


def test_lin_mirrors_mlx_ops(oracle, nqlib):
    """lin() infers bits from the shapes exactly as mlx_ops::lin does, and
    serves a layer stored without scales as matmul(x, W^T)."""
    import neurons_b200 as nb
    rng = np.random.default_rng(3)
    for bits in (4, 8):
        wq, s, b = oracle.quantize(weights(rng, 64, 512), bits, 64, 0)
        wm = {"q_proj.weight": dev_u32(wq), "q_proj.scales": dev_bf16(s),
              "q_proj.biases": dev_bf16(b)}
        x = acts(rng, 3, 512)
        y = nb.lin(dev_bf16(x), "q_proj", wm, 64)
        assert_close(host_u16(y), oracle.qmm(x, wq, s, b, bits, 64), f"lin bits={bits}")
    # a layer without scales is a plain matmul, as in mlx_ops::lin and the C++
    # cuda_ops::lin (same reference and tolerance as the C++ dense test)
    w = oracle.f32_to_bf16(weights(rng, 96, 512))
    y = nb.lin(dev_bf16(x), "dense", {"dense.weight": dev_bf16(w)}, 64)
    ref = oracle.bf16_to_f32(x).astype(np.float64) @ oracle.bf16_to_f32(w).astype(np.float64).T
    assert_close(host_u16(y), oracle.f32_to_bf16(ref.astype(np.float32)), "dense lin")


def test_back_to_back_launches_are_ordered(oracle, nqlib):
    """Programmatic dependent launch must not let a projection read an input the
    previous projection is still writing: chain y1 = W1 x, y2 = W2 y1."""
    import neurons_b200 as nb
    rng = np.random.default_rng(9)
    w1 = oracle.quantize(weights(rng, 512, 512), 4, 64, 0)
    w2 = oracle.quantize(weights(rng, 512, 512), 4, 64, 0)
    x = acts(rng, 1, 512)
    d1 = [dev_u32(w1[0]), dev_bf16(w1[1]), dev_bf16(w1[2])]
    d2 = [dev_u32(w2[0]), dev_bf16(w2[1]), dev_bf16(w2[2])]
    xd = dev_bf16(x)
    for _ in range(20):
        y1 = nb.quantized_matmul(xd, *d1, True, 64, 4)
        y2 = nb.quantized_matmul(y1, *d2, True, 64, 4)
    assert_close(host_u16(y1), oracle.qmm(x, *w1, 4, 64), "chained stage 1")
    ref2 = oracle.qmm(host_u16(y1), *w2, 4, 64)
    assert_close(host_u16(y2), ref2, "chained stage 2")


@pytest.mark.parametrize("N,K", [(14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_mistral_mlp_sweep(oracle, nqlib, N, K, bits, gs):
    """The parameter sweep on Mistral-7B MLP shapes (up 4096 -> 14336 and down
    14336 -> 4096) at every bit width, group size and M in {1, 8, 32, 128, 512,
    2048}: GEMV and tensor-core paths, seeded N(0, 0.02) weights quantized on the
    device (MLX affine scheme) and N(0, 1) activations.  Every output of 48
    sampled weight rows is checked against the oracle's matmul of the same
    codes."""
    import neurons_b200 as nb
    g = torch.Generator(device="cuda").manual_seed(N + K + bits + gs)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.02
    wq, s, b = nb.quantize(w, gs, bits, nb.SCHEME_MLX_AFFINE)
    del w
    rows = np.sort(np.random.default_rng(bits * gs).choice(N, 48, replace=False))
    wq_h = wq.cpu().view(torch.int32).numpy().view(np.uint32)[rows]
    s_h, b_h = host_u16(s)[rows], host_u16(b)[rows]
    for M in (1, 8, 32, 128, 512, 2048):
        x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        y = nb.quantized_matmul(x, wq, s, b, True, gs, bits)
        torch.cuda.synchronize()
        assert nb.take_device_error() == 0
        ref = oracle.qmm(host_u16(x), wq_h, s_h, b_h, bits, gs)
        assert_close(host_u16(y)[:, rows], ref, f"mistral {N}x{K} b{bits} g{gs} M={M}")


@pytest.mark.parametrize("M", [1, 2, 5, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("N,K", [(16, 1024), (100, 2048), (3072, 3072), (1000, 4096), (40, 8192),
                                 (33, 6144)])
def test_row_group_gemv(oracle, nqlib, M, gs, N, K):
    """The row-group decode kernel (4-bit, M <= 8, K a multiple of 128 split
    exactly over 4..16 warps): ragged row counts, every group size, and slice
    lengths of 2, 3, 4 and 8 k-blocks."""
    run_case(oracle, M, N, K, 4, gs, seed=N + K + M + gs)


def test_row_group_gemv_many_rows(oracle, nqlib):
    """More row groups than 8 per SM: the long-slice configuration (LM-head
    sized, here 20000 x 3072) with sampled rows against the oracle."""
    import neurons_b200 as nb
    rng = np.random.default_rng(20000)
    N, K = 20000, 3072
    wq, s, b = oracle.quantize(weights(rng, N, K), 4, 64, 1)
    x = acts(rng, 3, K)
    y = host_u16(nb.quantized_matmul(dev_bf16(x), dev_u32(wq), dev_bf16(s), dev_bf16(b), True,
                                      64, 4))
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    rows = np.sort(rng.choice(N, 256, replace=False))
    assert_close(y[:, rows], oracle.qmm(x, wq[rows], s[rows], b[rows], 4, 64), "20000x3072")
    assert_close(y[:, -16:], oracle.qmm(x, wq[-16:], s[-16:], b[-16:], 4, 64), "last rows")


@pytest.mark.parametrize("N,M", [(16400, 1), (16400, 8), (16384, 2)])
def test_row_group_gemv_paired_groups(oracle, nqlib, N, M):
    """Two row groups per CTA, the second staged by bulk copies into shared
    memory (shapes whose single-group CTAs do not fit one wave, here about
    the decode step's gate|up).  N = 16400: the last CTA's second group lies
    past the end and must store nothing; every row at the ragged end is
    checked."""
    import neurons_b200 as nb
    rng = np.random.default_rng(N + M)
    K = 3072
    wq, s, b = oracle.quantize(weights(rng, N, K), 4, 64, 0)
    x = acts(rng, M, K)
    y = host_u16(nb.quantized_matmul(dev_bf16(x), dev_u32(wq), dev_bf16(s), dev_bf16(b), True,
                                      64, 4))
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    rows = np.sort(rng.choice(N, 256, replace=False))
    assert_close(y[:, rows], oracle.qmm(x, wq[rows], s[rows], b[rows], 4, 64), f"{N}x{K} M={M}")
    assert_close(y[:, -48:], oracle.qmm(x, wq[-48:], s[-48:], b[-48:], 4, 64), "last rows")


def test_row_group_gemv_chained_launches(oracle, nqlib):
    """Back-to-back row-group launches under programmatic dependent launch:
    y2 = W2 y1 right after y1 = W1 x (the second kernel's weight loads run
    ahead, its activation reads must wait for the first kernel)."""
    import neurons_b200 as nb
    rng = np.random.default_rng(4096)
    w1 = oracle.quantize(weights(rng, 4096, 3072), 4, 64, 0)
    w2 = oracle.quantize(weights(rng, 3072, 4096), 4, 64, 0)
    x = acts(rng, 2, 3072)
    d1 = [dev_u32(w1[0]), dev_bf16(w1[1]), dev_bf16(w1[2])]
    d2 = [dev_u32(w2[0]), dev_bf16(w2[1]), dev_bf16(w2[2])]
    xd = dev_bf16(x)
    for _ in range(20):
        y1 = nb.quantized_matmul(xd, *d1, True, 64, 4)
        y2 = nb.quantized_matmul(y1, *d2, True, 64, 4)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    assert_close(host_u16(y1), oracle.qmm(x, *w1, 4, 64), "row-group chain stage 1")
    assert_close(host_u16(y2), oracle.qmm(host_u16(y1), *w2, 4, 64), "row-group chain stage 2")
