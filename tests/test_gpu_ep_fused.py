"""The all-to-all expert-parallel switch step (nq_ep_moe_switch_fused) with a
communicator of one rank on one GPU: every token is sent to this rank, its
flags are set by its own kernels (no wait depends on another process), and
the result must equal the single-GPU switch step nq_moe_switch wherever both
group the pairs by expert -- the same kernels, the same fp32 sums over the
same slots in the same order -- agree with it normwise where it takes its
few-token kernels, and match the oracle normwise.  Shapes: the Qwen3-30B-A3B
layer dims (E=128, top-8, H=2048, I=768, 4-bit g64)."""
import numpy as np
import pytest
import torch

from _util import acts, assert_close, dev_bf16, dev_f32, dev_i32, dev_u32, host_u16, weights

pytestmark = pytest.mark.gpu


def _experts(oracle, rng, E, rows, cols):
    wq, s, b = oracle.quantize(weights(rng, E * rows, cols), 4, 64, 0)
    host = (wq.reshape(E, rows, -1), s.reshape(E, rows, -1), b.reshape(E, rows, -1))
    return host, (dev_u32(host[0]), dev_bf16(host[1]), dev_bf16(host[2]))


@pytest.fixture(scope="module")
def comm1():
    from neurons_b200 import dist
    c = dist.Comm()
    c.symmetric_alloc(64 << 20)
    yield c
    c.close()


@pytest.mark.parametrize("T,fused_combine", [(1, "0"), (20, "0"), (300, "0"), (300, "1")])
def test_ep_fused_one_rank_equals_switch(oracle, nqlib, comm1, monkeypatch, T, fused_combine):
    """fused_combine "1": the combine folded into the down kernel writes the
    returned rows (NQ_MOE_FUSED_COMBINE)."""
    import neurons_b200 as nb
    from neurons_b200 import dist
    monkeypatch.setenv("NQ_MOE_FUSED_COMBINE", fused_combine)
    E, k, H, I = 128, 8, 2048, 768
    rng = np.random.default_rng(700 + T)
    (gh, gd), (uh, ud), (dh, dd) = (_experts(oracle, rng, E, I, H), _experts(oracle, rng, E, I, H),
                                    _experts(oracle, rng, E, H, I))
    assert dist.ep_fused_arena_size(T, k, H, 1) <= 64 << 20
    for call in range(3):  # repeated calls: epochs advance, buffers are reused
        x = acts(rng, T, H)
        idx, sc = oracle.moe_route(acts(rng, T, E), k)
        xd, idxd, scd = dev_bf16(x), dev_i32(idx), dev_f32(sc)
        ref = nb.moe_switch(xd, idxd, scd, gd, ud, dd)
        y = dist.ep_moe_switch_fused(comm1, xd, T, idxd, scd, gd, ud, dd, E, 0)
        torch.cuda.synchronize()
        assert nb.take_device_error() == 0 and comm1.take_error() == 0
        if T * k > E:  # both group the pairs by expert: the same kernels
            assert torch.equal(y, ref), f"T={T} call {call}: differs from nq_moe_switch"
        else:
            # nq_moe_switch takes its few-token kernels here, the expert shard
            # always groups: two different roundings of the two-stage step, so
            # they agree end to end (normwise), as each agrees with the oracle
            yy, rr = y.float(), ref.float()
            assert float((yy - rr).norm() / rr.norm()) < 1e-2, f"T={T} call {call}"
        if call == 0:
            r = oracle.moe_switch(x, idx, sc, (gh[0], gh[1], gh[2]), (uh[0], uh[1], uh[2]),
                                  (dh[0], dh[1], dh[2]), 4, 64, rounding=1)
            yy = oracle.bf16_to_f32(host_u16(y)).astype(np.float64)
            rr = oracle.bf16_to_f32(r).astype(np.float64)
            assert np.linalg.norm(yy - rr) / np.linalg.norm(rr) < 1e-2


def test_ep_fused_rejects_before_enqueueing(nqlib, comm1):
    """A rejected call (arena region out of range) launches nothing: the
    communicator's call count is unchanged, so a following call still works."""
    import neurons_b200 as nb
    from neurons_b200 import dist
    E, k, H, I, T = 16, 4, 256, 128, 8
    g = torch.Generator(device="cuda").manual_seed(1)
    W = [nb.quantize(torch.randn(E, n, kk, device="cuda", generator=g) * 0.02)
         for n, kk in ((I, H), (I, H), (H, I))]
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    idx, sc = nb.moe_route(torch.randn(T, E, device="cuda", generator=g).to(torch.bfloat16), k)
    with pytest.raises(nb.NQError):
        dist.ep_moe_switch_fused(comm1, x, T, idx, sc, *W, E, (64 << 20) - 256)
    y = dist.ep_moe_switch_fused(comm1, x, T, idx, sc, *W, E, 0)
    ref = nb.moe_switch(x, idx, sc, *W)
    torch.cuda.synchronize()
    assert comm1.take_error() == 0 and torch.equal(y, ref)
