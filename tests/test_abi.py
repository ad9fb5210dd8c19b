"""CPU tests of the C ABI: the library loads, exports every entry point that
include/nq.h declares, and validates arguments (status codes mirror
compute::ErrorCode) before touching a device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nq.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nq_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("nq_quantized_matmul", "nq_dequantize", "nq_quantize", "nq_gather_qmm",
                 "nq_moe_route", "nq_moe_switch", "nq_bits_from_shapes"):
        assert name in syms


def test_library_exports_every_declared_symbol(nqlib):
    for name in declared_symbols():
        assert hasattr(nqlib, name), name


def test_python_signatures_cover_header():
    from neurons_b200._lib import SIGNATURES
    assert sorted(SIGNATURES) == declared_symbols()


def test_version_and_device_count(nqlib):
    assert nqlib.nq_version() >= 1
    assert nqlib.nq_device_count() >= 0


@pytest.mark.parametrize("w_cols,s_cols,gs", [(512, 64, 64), (1024, 64, 64), (96, 12, 64),
                                              (192, 12, 64), (0, 64, 64), (1024, 32, 128)])
def test_bits_from_shapes_matches_oracle(nqlib, oracle, w_cols, s_cols, gs):
    assert nqlib.nq_bits_from_shapes(w_cols, s_cols, gs) == \
        oracle.bits_from_shapes(w_cols, s_cols, gs)


DUMMY = ctypes.c_void_p(16)  # never dereferenced: validation fails first


@pytest.mark.parametrize("bits,gs,K", [(3, 64, 128), (4, 48, 96), (4, 64, 96), (8, 16, 64)])
def test_qmm_rejects_bad_quant_params(nqlib, bits, gs, K):
    rc = nqlib.nq_quantized_matmul(DUMMY, 1, DUMMY, DUMMY, DUMMY, 8, K, bits, gs, DUMMY, None)
    assert rc == 1  # InvalidInput
    assert nqlib.nq_last_error()


def test_qmm_requires_biases(nqlib):
    rc = nqlib.nq_quantized_matmul(DUMMY, 1, DUMMY, DUMMY, None, 8, 64, 4, 64, DUMMY, None)
    assert rc == 1
    assert b"biases" in nqlib.nq_last_error()


def test_qmm_rejects_unaligned(nqlib):
    rc = nqlib.nq_quantized_matmul(ctypes.c_void_p(18), 1, DUMMY, DUMMY, DUMMY, 8, 64, 4, 64,
                                   DUMMY, None)
    assert rc == 1
    assert b"aligned" in nqlib.nq_last_error()


def test_empty_shapes_are_noops(nqlib):
    assert nqlib.nq_quantized_matmul(None, 0, None, None, None, 8, 64, 4, 64, None, None) == 0
    assert nqlib.nq_dequantize(None, None, None, 0, 64, 4, 64, None, None) == 0
    assert nqlib.nq_moe_route(None, 0, 128, 8, None, None, None) == 0


def test_launch_count_query_validates(nqlib):
    assert nqlib.nq_quantized_matmul_launches(0, 4096, 4096, 4, 64) == 0
    assert nqlib.nq_quantized_matmul_launches(8, 0, 4096, 4, 64) == 0
    assert nqlib.nq_quantized_matmul_launches(8, 64, 96, 4, 64) == 1  # K % group_size
    assert nqlib.nq_quantized_matmul_launches(-1, 64, 128, 4, 64) == 1


def test_gather_rejects_bad_batch(nqlib):
    rc = nqlib.nq_gather_qmm(DUMMY, 3, 1, None, DUMMY, 8, DUMMY, DUMMY, DUMMY, 16, 32, 64, 4, 32,
                             DUMMY, None)
    assert rc == 1


def test_moe_rejects_bad_topk(nqlib):
    assert nqlib.nq_moe_route(DUMMY, 4, 128, 0, DUMMY, DUMMY, None) == 1
    assert nqlib.nq_moe_route(DUMMY, 4, 4, 8, DUMMY, DUMMY, None) == 1
    assert nqlib.nq_moe_route(DUMMY, 4, 2048, 8, DUMMY, DUMMY, None) == 1


def test_moe_workspace_too_small(nqlib):
    need = nqlib.nq_moe_workspace_size(64, 128, 8, 2048, 768)
    assert need > 64 * 8 * 768 * 2
    rc = nqlib.nq_moe_switch(DUMMY, 64, 2048, 768, 128, 8, DUMMY, DUMMY, DUMMY, DUMMY, DUMMY,
                             DUMMY, DUMMY, DUMMY, DUMMY, DUMMY, DUMMY, 4, 64, DUMMY, need - 1,
                             DUMMY, None)
    assert rc == 1
    assert b"workspace" in nqlib.nq_last_error()


def test_no_device_is_backend_not_available(nqlib):
    if nqlib.nq_device_count() > 0:
        pytest.skip("a CUDA device is present")
    rc = nqlib.nq_quantized_matmul(DUMMY, 1, DUMMY, DUMMY, DUMMY, 8, 64, 4, 64, DUMMY, None)
    assert rc == 3  # BackendNotAvailable


def test_python_errors_carry_error_code():
    import torch
    from neurons_b200 import NQError, quantized_matmul
    with pytest.raises(NQError) as ei:
        quantized_matmul(torch.zeros(1, 64, dtype=torch.bfloat16), None, None)
    assert ei.value.code == "InvalidInput"


class NqPush(__import__("ctypes").Structure):
    """nq_push_t (include/nq.h)."""
    import ctypes as _c
    _fields_ = [("nranks", _c.c_int), ("rank", _c.c_int), ("epoch", _c.c_void_p),
                ("dst", _c.c_void_p * 8), ("ready", _c.c_void_p)]


def test_push_check_names_misaligned_scales(nqlib):
    """A fused tensor-parallel call whose scale shard is not 16-byte aligned is
    rejected by the check that runs before the call enqueues anything (its
    ready kernel included), and the message names the scales.  Pointers are
    never dereferenced by the check, so this needs no device."""
    import ctypes
    p = NqPush()
    p.nranks, p.rank, p.epoch, p.ready = 2, 0, 0x5000, 0x6000
    p.dst[0], p.dst[1] = 0x7000, 0x8000
    args = [ctypes.c_void_p(0x1000), 1, ctypes.c_void_p(0x2000), ctypes.c_void_p(0x3002),
            ctypes.c_void_p(0x4000), 64, 512, 4, 64, 128, 0, ctypes.byref(p)]
    rc = nqlib.nq_quantized_matmul_push_check(*args)
    assert rc == 1, rc  # NQ_INVALID_INPUT
    assert b"scales and biases must be 16-byte aligned" in nqlib.nq_last_error()
    args[3] = ctypes.c_void_p(0x3000)
    args[10] = 100  # columns [100, 164) outside N_total = 128
    assert nqlib.nq_quantized_matmul_push_check(*args) == 1
    assert b"columns outside" in nqlib.nq_last_error()


def test_llama_create_validates_on_the_host(nqlib):
    """nq_llama_create rejects NULL arguments and configurations the decode
    step does not serve before it touches a device."""
    import ctypes
    from neurons_b200.llama import LlamaConfig, LlamaLayer, QWeight
    out = ctypes.c_void_p()
    assert nqlib.nq_llama_create(ctypes.byref(out), None, None, None, None, None) == 1
    cfg = LlamaConfig(n_layers=1, hidden=3072, n_heads=24, n_kv_heads=8, head_dim=128,
                      intermediate=8192, vocab=1000, bits=8, group_size=64, max_context=16,
                      rms_eps=1e-5, rope_theta=1e4)
    layers = (LlamaLayer * 1)()
    dummy = ctypes.c_void_p(256)
    emb = QWeight(dummy, dummy, dummy)
    rc = nqlib.nq_llama_create(ctypes.byref(out), ctypes.byref(cfg), layers, dummy,
                               ctypes.byref(emb), None)
    assert rc == 1 and b"4-bit" in nqlib.nq_last_error()
    cfg.bits, cfg.n_kv_heads = 4, 5  # 24 heads do not split over 5 KV heads
    rc = nqlib.nq_llama_create(ctypes.byref(out), ctypes.byref(cfg), layers, dummy,
                               ctypes.byref(emb), None)
    assert rc == 1 and b"n_kv_heads" in nqlib.nq_last_error()
    cfg.n_kv_heads, cfg.hidden = 8, 320  # K = 320 is not served by the decode GEMV
    rc = nqlib.nq_llama_create(ctypes.byref(out), ctypes.byref(cfg), layers, dummy,
                               ctypes.byref(emb), None)
    assert rc == 1
    assert not out.value
