"""Failure detection on the device, in the form that faults no GPU: every wait
inside the kernels is bounded (2 s of %globaltimer).  A fused tensor-parallel
compute step is given two ranks whose second ready flag nothing ever sets; the
kernel's storing warps give up after the limit, store nothing, raise the
timeout bit of the device error word and return, so the call completes and the
context stays usable (a following call computes correctly)."""
import ctypes

import numpy as np
import pytest
import torch

from _util import acts, assert_close, dev_bf16, dev_u32, host_u16, weights

pytestmark = pytest.mark.gpu

ERR_WAIT_TIMEOUT = 1  # nq DeviceError kErrWaitTimeout


class NqPush(ctypes.Structure):
    """nq_push_t (include/nq.h)."""
    _fields_ = [("nranks", ctypes.c_int), ("rank", ctypes.c_int), ("epoch", ctypes.c_void_p),
                ("dst", ctypes.c_void_p * 8), ("ready", ctypes.c_void_p)]


@pytest.mark.parametrize("M", [1, 64])
def test_push_wait_times_out_and_gpu_stays_usable(oracle, nqlib, M):
    import neurons_b200 as nb
    rng = np.random.default_rng(M)
    N, K = 256, 512
    wq, s, b = oracle.quantize(weights(rng, N, K), 4, 64, 0)
    x = acts(rng, M, K)
    d = [dev_bf16(x), dev_u32(wq), dev_bf16(s), dev_bf16(b)]
    epoch = torch.ones(1, dtype=torch.int32, device="cuda")
    ready = torch.tensor([1, 0], dtype=torch.int32, device="cuda")  # rank 1 never signals
    y = [torch.zeros(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    p = NqPush()
    p.nranks, p.rank = 2, 0
    p.epoch, p.ready = epoch.data_ptr(), ready.data_ptr()
    p.dst[0], p.dst[1] = y[0].data_ptr(), y[1].data_ptr()
    nb.take_device_error()
    torch.cuda.synchronize()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = nqlib.nq_quantized_matmul_push(ptr(d[0]), M, ptr(d[1]), ptr(d[2]), ptr(d[3]), N, K, 4,
                                        64, N, 0, ctypes.byref(p), st)
    assert rc == 0, nqlib.nq_last_error()
    torch.cuda.synchronize()  # returns: the waits are bounded
    assert nb.take_device_error() & ERR_WAIT_TIMEOUT
    assert not y[0].any() and not y[1].any(), "no store after a failed ready wait"
    # the context is intact: the same product through the ordinary call
    out = nb.quantized_matmul(d[0], d[1], d[2], d[3], True, 64, 4)
    torch.cuda.synchronize()
    assert nb.take_device_error() == 0
    assert_close(host_u16(out), oracle.qmm(x, wq, s, b, 4, 64), f"after timeout M={M}")
