"""nq_moe_switch_static: the MoE switch step for callers that cannot allocate.

Some hosts of this library cannot call cudaMalloc themselves -- an FFI
binding or a runtime that only passes in the tensors it already owns, with
no allocator of its own to hand over.  nq_moe_switch_static serves them: it
takes the same arguments as nq_moe_switch minus the workspace and draws its
scratch from a fixed block inside the library.

This file is named so that pytest collects it after every other test file.
It must pass both on its own in a fresh process (the first call on the
device performs the block's address lookup) and after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

from _util import (acts, assert_close, dev_bf16, dev_f32, dev_i32, dev_u32, host_u16, weights,
                   workspace_hidden)

pytestmark = pytest.mark.gpu


def _experts(oracle, rng, E, rows, cols):
    """(host, device) copies of E stacked quantized experts."""
    wq, s, b = oracle.quantize(weights(rng, E * rows, cols), 4, 64, 0)
    host = (wq.reshape(E, rows, -1), s.reshape(E, rows, -1), b.reshape(E, rows, -1))
    return host, (dev_u32(host[0]), dev_bf16(host[1]), dev_bf16(host[2]))


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _call_static(lib, x, idx, sc, gate, up, down, y):
    T, H = x.shape
    E, I = gate[0].shape[0], gate[0].shape[1]
    k = idx.shape[1]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.nq_moe_switch_static(_p(x), T, H, I, E, k, _p(idx), _p(sc),
                                    _p(gate[0]), _p(gate[1]), _p(gate[2]),
                                    _p(up[0]), _p(up[1]), _p(up[2]),
                                    _p(down[0]), _p(down[1]), _p(down[2]),
                                    4, 64, _p(y), stream)


def _call_workspace(lib, x, idx, sc, gate, up, down, y):
    T, H = x.shape
    E, I = gate[0].shape[0], gate[0].shape[1]
    k = idx.shape[1]
    need = lib.nq_moe_workspace_size(T, E, k, H, I)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.nq_moe_switch(_p(x), T, H, I, E, k, _p(idx), _p(sc),
                           _p(gate[0]), _p(gate[1]), _p(gate[2]),
                           _p(up[0]), _p(up[1]), _p(up[2]),
                           _p(down[0]), _p(down[1]), _p(down[2]),
                           4, 64, _p(ws), need, _p(y), stream)
    return rc, ws


@pytest.mark.parametrize("T", [1, 20])
def test_static_scratch_matches_workspace_entry_point(oracle, nqlib, T):
    """Two calls in a row on different token batches (T=1: one problem per pair;
    T=20: pairs grouped by expert, which needs zeroed counters), each checked
    against nq_moe_switch with a caller-provided workspace, at the Qwen3-30B-A3B
    layer dims (E=128, top-8, hidden 2048, intermediate 768, 4-bit g64).  The
    first call is also held to the oracle stage by stage: the SwiGLU activations
    h (read from the workspace call, which runs the same kernels on the same
    inputs) against the oracle's first stage, and the static call's y against
    the oracle's second stage applied to that h."""
    E, k, H, I = 128, 8, 2048, 768
    rng = np.random.default_rng(100 + T)
    (gate_h, gate), (up_h, up), (down_h, down) = (
        _experts(oracle, rng, E, I, H), _experts(oracle, rng, E, I, H),
        _experts(oracle, rng, E, H, I))
    for call in range(2):
        x = acts(rng, T, H)
        idx, sc = oracle.moe_route(acts(rng, T, E), k)
        xd, idxd, scd = dev_bf16(x), dev_i32(idx), dev_f32(sc)
        y_static = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device="cuda")
        y_ws = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
        assert _call_static(nqlib, xd, idxd, scd, gate, up, down, y_static) == 0, \
            nqlib.nq_last_error()
        rc, ws = _call_workspace(nqlib, xd, idxd, scd, gate, up, down, y_ws)
        assert rc == 0, nqlib.nq_last_error()
        torch.cuda.synchronize()
        err = ctypes.c_uint(0)
        assert nqlib.nq_take_device_error(ctypes.byref(err)) == 0 and err.value == 0
        assert_close(host_u16(y_static), host_u16(y_ws), f"static vs workspace, call {call}")
        if call == 0:
            h = workspace_hidden(ws, T, E, k, H, I)
            assert_close(h, oracle.moe_hidden(x, idx, gate_h, up_h, 4, 64, rounding=1),
                         f"T={T} h vs oracle")
            assert_close(host_u16(y_static),
                         oracle.moe_combine(h, idx, sc, down_h, 4, 64, rounding=1),
                         f"T={T} static y vs oracle")


def test_static_scratch_rejects_oversize(nqlib):
    """A call whose scratch would not fit the static block fails cleanly."""
    E, k, H, I, T = 128, 8, 2048, 768, 4096
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    p = _p(dummy)
    rc = nqlib.nq_moe_switch_static(p, T, H, I, E, k, p, p, p, p, p, p, p, p, p, p, p, 4, 64, p,
                                    None)
    assert rc == 1  # NQ_INVALID_INPUT
    assert b"static scratch" in nqlib.nq_last_error()
