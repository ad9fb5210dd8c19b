"""Decode-step replay of LlamaModel's lin() sequence (llama_model.cpp:393-494):
every projection of the last layer and the LM head checked against the oracle
on the GPU's own inputs, and a CUDA-graph replay of the step checked against
the eager step bit for bit."""
import numpy as np
import pytest
import torch

from _util import assert_close, host_u16, host_u32

pytestmark = pytest.mark.gpu


def _oracle_lin(oracle, rp, x, key):
    wm = rp.wm
    return oracle.qmm(host_u16(x), host_u32(wm[key + ".weight"]), host_u16(wm[key + ".scales"]),
                      host_u16(wm[key + ".biases"]), rp.bits, rp.gs)


@pytest.mark.parametrize("bits,gs", [(4, 64), (8, 32)])
def test_replay_projections_match_oracle(oracle, nqlib, bits, gs):
    from neurons_b200.replay import LlamaDecodeReplay
    rp = LlamaDecodeReplay(hidden=256, n_heads=4, n_kv=2, head_dim=64, inter=768, layers=2,
                           vocab=1000, bits=bits, group_size=gs, seed=3)
    g = torch.Generator(device="cuda").manual_seed(1)
    rp.x.copy_(torch.randn(rp.x.shape, device="cuda", generator=g).to(torch.bfloat16))
    rp.step()
    torch.cuda.synchronize()
    last = f"model.layers.{rp.layers - 1}."
    checks = [(rp.q, rp.o, last + "self_attn.o_proj"),
              (rp.o, rp.gate, last + "mlp.gate_proj"),
              (rp.o, rp.up, last + "mlp.up_proj"),
              (rp.gate, rp.h, last + "mlp.down_proj"),
              (rp.h, rp.logits, "lm_head")]
    for inp, out, key in checks:
        assert_close(host_u16(out), _oracle_lin(oracle, rp, inp, key), key)


def test_replay_graph_matches_eager(nqlib):
    from neurons_b200.replay import LlamaDecodeReplay
    import neurons_b200 as nb
    rp = LlamaDecodeReplay(hidden=512, n_heads=8, n_kv=2, head_dim=64, inter=1536, layers=3,
                           vocab=4096, seed=5)
    assert rp.launches_per_token() == 22
    g = torch.Generator(device="cuda").manual_seed(2)
    rp.x.copy_(torch.randn(rp.x.shape, device="cuda", generator=g).to(torch.bfloat16))
    rp.step()
    torch.cuda.synchronize()
    eager = rp.logits.clone()
    rp.logits.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        rp.step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    assert torch.equal(rp.logits.view(torch.int16), eager.view(torch.int16))
    assert np.isfinite(rp.logits.float().cpu().numpy()).all()
