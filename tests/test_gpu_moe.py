"""GPU parity: gather_qmm, the MoE router and the batched switch step through
the C ABI against the oracle (Qwen3-30B-A3B layer dims: E=128, top-8,
hidden 2048, moe_intermediate 768, 4-bit g64)."""
import os

import numpy as np
import pytest
import torch

from _util import (acts, assert_close, dev_bf16, dev_f32, dev_i32, dev_u32, host_u16,
                   weights, workspace_hidden)

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def experts(oracle, rng, E, rows, cols, bits=4, gs=64):
    wq, s, b = oracle.quantize(weights(rng, E * rows, cols), bits, gs, 0)
    return wq.reshape(E, rows, -1), s.reshape(E, rows, -1), b.reshape(E, rows, -1)


def dev3(t):
    return dev_u32(t[0]), dev_bf16(t[1]), dev_bf16(t[2])


def test_golden_gather(nqlib):
    import neurons_b200 as nb
    g = np.load(os.path.join(GOLDEN, "seeded_small.npz"))
    out = nb.gather_qmm(dev_bf16(g["gq_x"]), dev_u32(g["moe_gate_wq"]), dev_bf16(g["moe_gate_s"]),
                        dev_bf16(g["moe_gate_b"]), None, dev_i32(g["gq_rhs"]), True, 32, 4)
    assert_close(host_u16(out), g["gq_out"], "golden gather")


def test_gather_decode_shape(oracle, nqlib):
    """x [1, 2048] against 8 of 128 experts [768, 2048] (the reference's decode call)."""
    import neurons_b200 as nb
    rng = np.random.default_rng(0)
    W = experts(oracle, rng, 128, 768, 2048)
    x = acts(rng, 1, 2048)[None]
    rhs = rng.choice(128, 8, replace=False).astype(np.int32)
    out = nb.gather_qmm(dev_bf16(x), *dev3(W), None, dev_i32(rhs), True, 64, 4)
    ref = oracle.gather_qmm(x, *W, rhs, bits=4, group_size=64)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    for i in range(8):
        r = oracle.qmm(x[0], W[0][rhs[i]], W[1][rhs[i]], W[2][rhs[i]], 4, 64)
        assert_close(host_u16(out)[i], r, f"slot {i}")
    assert_close(host_u16(out), ref, "gather vs oracle bf16")


def test_gather_batched_x_and_lhs(oracle, nqlib):
    import neurons_b200 as nb
    rng = np.random.default_rng(1)
    W = experts(oracle, rng, 6, 40, 256, 8, 32)
    x = acts(rng, 4 * 3, 256).reshape(4, 3, 256)       # x_batch 4, M 3
    rhs = np.array([5, 0, 3, 3], np.int32)
    out = nb.gather_qmm(dev_bf16(x), *dev3(W), None, dev_i32(rhs), True, 32, 8)
    ref = oracle.gather_qmm(x, *W, rhs, bits=8, group_size=32)
    assert_close(host_u16(out), ref, "x_batch == n_idx")
    lhs = np.array([2, 2, 0, 1, 3], np.int32)
    rhs2 = np.array([1, 4, 4, 0, 5], np.int32)
    out2 = nb.gather_qmm(dev_bf16(x), *dev3(W), dev_i32(lhs), dev_i32(rhs2), True, 32, 8)
    ref2 = oracle.gather_qmm(x, *W, rhs2, lhs=lhs, bits=8, group_size=32)
    assert_close(host_u16(out2), ref2, "lhs indices")


def test_gather_bad_index_zeroes_and_flags(oracle, nqlib):
    import neurons_b200 as nb
    rng = np.random.default_rng(2)
    W = experts(oracle, rng, 4, 32, 128, 4, 32)
    x = acts(rng, 1, 128)[None]
    nb.take_device_error()
    out = nb.gather_qmm(dev_bf16(x), *dev3(W), None, dev_i32(np.array([1, 9], np.int32)),
                        True, 32, 4)
    torch.cuda.synchronize()
    assert nb.take_device_error() & 2
    assert (host_u16(out)[1] == 0).all()
    ref = oracle.gather_qmm(x, *W, np.array([1], np.int32), bits=4, group_size=32)
    assert_close(host_u16(out)[:1], ref, "valid slot")


@pytest.mark.parametrize("T", [1, 7, 64, 2048])
def test_route_matches_oracle(oracle, nqlib, T):
    import neurons_b200 as nb
    rng = np.random.default_rng(T)
    logits = acts(rng, T, 128)
    idx, sc = nb.moe_route(dev_bf16(logits), 8)
    ridx, rsc = oracle.moe_route(logits, 8)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(sc.cpu().numpy(), rsc, rtol=2e-6, atol=1e-7)


def test_route_ties(oracle, nqlib):
    import neurons_b200 as nb
    logits = oracle.f32_to_bf16(np.array([[0.5, 1.0, 1.0, 0.25, 1.0] * 8], np.float32))
    idx, sc = nb.moe_route(dev_bf16(logits), 4)
    ridx, rsc = oracle.moe_route(logits, 4)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)


def staged_switch_check(oracle, x, idx, sc, gate, up, down, bits, gs, what):
    """The switch step is two matmul stages with a bf16 rounding between them
    (MLX rounds there too).  Each stage is held to the matmul tolerance on its own:
    h against the oracle's stage 1, and y against the oracle's stage 2 applied to
    the GPU's own h.  End to end, y must also match both the oracle's fused
    rounding points and MLX's op chain normwise."""
    import neurons_b200 as nb
    T, H = x.shape
    k = idx.shape[1]
    E, I = gate[0].shape[0], gate[0].shape[1]
    ws = torch.zeros(nb.moe_workspace_size(T, E, k, H, I), dtype=torch.uint8, device="cuda")
    y = nb.moe_switch(dev_bf16(x), dev_i32(idx), dev_f32(sc), dev3(gate), dev3(up), dev3(down),
                      gs, bits, workspace=ws)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    h_gpu = workspace_hidden(ws, T, E, k, H, I)
    assert_close(h_gpu, oracle.moe_hidden(x, idx, gate, up, bits, gs, rounding=1), what + " h")
    y_gpu = host_u16(y)
    assert_close(y_gpu, oracle.moe_combine(h_gpu, idx, sc, down, bits, gs, rounding=1),
                 what + " y")
    yy = oracle.bf16_to_f32(y_gpu).astype(np.float64)
    for rounding in (1, 0):
        r = oracle.bf16_to_f32(oracle.moe_switch(x, idx, sc, gate, up, down, bits, gs,
                                                 rounding=rounding)).astype(np.float64)
        assert np.linalg.norm(yy - r) / np.linalg.norm(r) < 1e-2, (what, rounding)


def test_golden_switch(oracle, nqlib):
    g = np.load(os.path.join(GOLDEN, "seeded_small.npz"))
    mats = [(g[f"moe_{n}_wq"], g[f"moe_{n}_s"], g[f"moe_{n}_b"]) for n in ("gate", "up", "down")]
    staged_switch_check(oracle, g["moe_x"], g["moe_idx"], g["moe_scores"], *mats, 4, 32,
                        "golden switch")


@pytest.mark.parametrize("T,E,k,H,I", [(1, 128, 8, 2048, 768), (20, 128, 8, 2048, 768),
                                       (64, 128, 8, 2048, 768), (512, 128, 8, 2048, 768),
                                       (3, 16, 4, 256, 128), (64, 16, 4, 256, 128),
                                       (100, 8, 2, 128, 64), (600, 4, 2, 256, 128)])
def test_switch_matches_oracle(oracle, nqlib, T, E, k, H, I):
    """pair mode (T*k <= E), grouped GEMV mode (E < T*k < 8 E) and the grouped
    tensor-core mode (T*k >= 8 E; (600, 4, 2) puts ~300 tokens on every expert,
    more than one 256-token tile)."""
    rng = np.random.default_rng(T * 31 + E)
    gate = experts(oracle, rng, E, I, H)
    up = experts(oracle, rng, E, I, H)
    down = experts(oracle, rng, E, H, I)
    x = acts(rng, T, H)
    idx, sc = oracle.moe_route(acts(rng, T, E), k)
    staged_switch_check(oracle, x, idx, sc, gate, up, down, 4, 64, f"switch T={T} E={E}")


@pytest.mark.parametrize("bits,gs", [(8, 32), (4, 128), (8, 64), (4, 32)])
def test_switch_tensor_core_bits_groups(oracle, nqlib, bits, gs):
    """The grouped tensor-core mode at every code width and group size."""
    T, E, k, H, I = 256, 16, 4, 256, 256
    rng = np.random.default_rng(bits * 100 + gs)
    gate = experts(oracle, rng, E, I, H, bits, gs)
    up = experts(oracle, rng, E, I, H, bits, gs)
    down = experts(oracle, rng, E, H, I, bits, gs)
    x = acts(rng, T, H)
    idx, sc = oracle.moe_route(acts(rng, T, E), k)
    staged_switch_check(oracle, x, idx, sc, gate, up, down, bits, gs,
                        f"switch {bits}-bit g{gs}")


@pytest.mark.parametrize("T", [20, 300])
def test_switch_partials_sum_to_the_full_step(oracle, nqlib, T):
    """Expert shards (the expert-parallel building block): the fp32 partials of
    four shards of 4 experts sum to the full switch step."""
    import neurons_b200 as nb
    E, k, H, I = 16, 4, 256, 128
    rng = np.random.default_rng(T)
    W = [experts(oracle, rng, E, r, c) for r, c in ((I, H), (I, H), (H, I))]
    x = acts(rng, T, H)
    idx, sc = oracle.moe_route(acts(rng, T, E), k)
    full = nb.moe_switch(dev_bf16(x), dev_i32(idx), dev_f32(sc), *(dev3(w) for w in W), 64, 4)
    tot = torch.zeros(T, H, dtype=torch.float32, device="cuda")
    for e0 in range(0, E, 4):
        sh = [tuple(a[e0:e0 + 4] for a in w) for w in W]
        tot += nb.moe_switch_partial(dev_bf16(x), dev_i32(idx), dev_f32(sc),
                                     *(dev3(w) for w in sh), E, e0, 64, 4)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    y = tot.to(torch.bfloat16)
    assert_close(host_u16(y), host_u16(full), f"partials T={T}")


def test_switch_qwen3_T2048_sampled_tokens(oracle, nqlib):
    """The benchmark's MoE layer at full size: Qwen3-30B-A3B dims (E=128, top-8,
    H=2048, I=768, 4-bit g64), T=2048 tokens on the grouped tensor-core path
    (about 128 tokens per expert, the busiest near 150; experts spanning more
    than one 256-token tile are covered by the (600, 4, 2) case above).  Tokens
    are independent given their routing, so a seeded sample of 64 tokens is
    checked stage by stage against the oracle (h of every sampled pair, y of
    every sampled token, and y end to end)."""
    import neurons_b200 as nb
    T, E, k, H, I = 2048, 128, 8, 2048, 768
    g = torch.Generator(device="cuda").manual_seed(2048)
    mats = []
    for rows, cols in ((I, H), (I, H), (H, I)):
        w = torch.randn(E, rows, cols, device="cuda", generator=g) * 0.02
        mats.append(nb.quantize(w, 64, 4, nb.SCHEME_MLX_AFFINE))
        del w
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, device="cuda", generator=g).to(torch.bfloat16)
    idx, sc = nb.moe_route(logits, k)
    ws = torch.zeros(nb.moe_workspace_size(T, E, k, H, I), dtype=torch.uint8, device="cuda")
    y = nb.moe_switch(x, idx, sc, *mats, 64, 4, workspace=ws)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    idx_h, sc_h = idx.cpu().numpy(), sc.cpu().numpy()
    assert np.bincount(idx_h.reshape(-1), minlength=E).min() > 0, "every expert is used"
    host = [(m[0].cpu().view(torch.int32).numpy().view(np.uint32), host_u16(m[1]),
             host_u16(m[2])) for m in mats]
    sample = np.sort(np.random.default_rng(0).choice(T, 64, replace=False))
    x_h = host_u16(x)[sample]
    h_all = workspace_hidden(ws, T, E, k, H, I).reshape(T, k, I)
    h_s = h_all[sample].reshape(-1, I)
    gate, up, down = host
    assert_close(h_s, oracle.moe_hidden(x_h, idx_h[sample], gate, up, 4, 64, rounding=1),
                 "T=2048 h (sampled pairs)")
    y_s = host_u16(y)[sample]
    assert_close(y_s, oracle.moe_combine(h_s, idx_h[sample], sc_h[sample], down, 4, 64,
                                         rounding=1), "T=2048 y (sampled tokens)")
    yy = oracle.bf16_to_f32(y_s).astype(np.float64)
    for rounding in (1, 0):
        r = oracle.bf16_to_f32(oracle.moe_switch(x_h, idx_h[sample], sc_h[sample], gate, up,
                                                 down, 4, 64, rounding=rounding))
        r = r.astype(np.float64)
        assert np.linalg.norm(yy - r) / np.linalg.norm(r) < 1e-2, rounding


@pytest.mark.parametrize("T", [512, 2048])
def test_fused_combine_matches_combine_kernel(oracle, nqlib, monkeypatch, T):
    """The score-weighted combine folded into the tensor-core down kernel
    (NQ_MOE_FUSED_COMBINE=1: the last pair of a token to land in an n-block
    sums the token's pairs in slot order) gives the same bits as the separate
    combine kernel, on two calls in a row (arrival counters reset), and the
    oracle's combine stage applied to the GPU's h."""
    import neurons_b200 as nb
    E, k, H, I = 128, 8, 2048, 768
    rng = np.random.default_rng(900 + T)
    gate, up, down = (experts(oracle, rng, E, I, H), experts(oracle, rng, E, I, H),
                      experts(oracle, rng, E, H, I))
    for call in range(2):
        x = acts(rng, T, H)
        idx, sc = oracle.moe_route(acts(rng, T, E), k)
        args = (dev_bf16(x), dev_i32(idx), dev_f32(sc), dev3(gate), dev3(up), dev3(down), 64, 4)
        monkeypatch.setenv("NQ_MOE_FUSED_COMBINE", "0")
        ref = nb.moe_switch(*args)
        monkeypatch.setenv("NQ_MOE_FUSED_COMBINE", "1")
        ws = torch.zeros(nb.moe_workspace_size(T, E, k, H, I), dtype=torch.uint8, device="cuda")
        y = nb.moe_switch(*args, workspace=ws)
        torch.cuda.synchronize()
        assert nb.take_device_error() == 0
        assert torch.equal(y, ref), f"T={T} call {call}"
        if call == 0:
            rows = np.random.default_rng(T).choice(T, 32, replace=False)
            h = workspace_hidden(ws, T, E, k, H, I).reshape(T, k, I)[rows].reshape(-1, I)
            assert_close(host_u16(y)[rows],
                         oracle.moe_combine(h, idx[rows], sc[rows], down, 4, 64, rounding=1),
                         f"T={T} fused combine vs oracle")
