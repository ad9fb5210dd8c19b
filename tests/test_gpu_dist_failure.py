"""Failure detection across ranks, on two GPUs, without a GPU fault: rank 1
stops making calls between steps (it stays alive and holds nothing in
flight), rank 0 makes the next tensor-parallel call and its bounded host
wait (nq_comm_wait, through nq_comm_set_timeout) must end it with an error
after the deadline, abort the NCCL communicator and leave the GPU usable.
NVLS is off (NCCL_NVLS_ENABLE=0) and no symmetric arena is mapped, so no
rank holds another's memory.  Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q, done):
    import sys
    import datetime
    import time
    sys.path.insert(0, ROOT)
    import torch.distributed as tdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    tdist.init_process_group("nccl", rank=rank, world_size=world,
                             timeout=datetime.timedelta(seconds=60),
                             device_id=torch.device("cuda", rank))
    out = {}
    try:
        import neurons_b200 as nb
        from neurons_b200 import dist
        comm = dist.Comm()
        comm.set_timeout(3000)
        g = torch.Generator(device="cuda").manual_seed(0)
        N, K = 1024, 512
        r0, rows = dist.tp_shard(N, world, rank)
        wq, s, b = nb.quantize(torch.randn(rows, K, device="cuda", generator=g) * 0.02, 64, 4)
        x = torch.randn(1, K, device="cuda", generator=g).to(torch.bfloat16)
        # step 1: every rank takes part
        y = dist.tp_quantized_matmul(comm, x, wq, s, b, N)
        out["step1"] = bool(torch.isfinite(y.float()).all())
        if rank == 0:
            # step 2: rank 1 is gone; the call must end by the deadline
            t0 = time.time()
            try:
                dist.tp_quantized_matmul(comm, x, wq, s, b, N)
                out["step2"] = "returned"
            except nb.NQError as e:
                out["step2"] = str(e)
            out["seconds"] = time.time() - t0
            # the communicator is unusable now, the GPU is not
            try:
                dist.tp_quantized_matmul(comm, x, wq, s, b, N)
                out["after"] = "returned"
            except nb.NQError as e:
                out["after"] = str(e)
            z = torch.ones(1024, device="cuda") * 2
            torch.cuda.synchronize()
            out["gpu_ok"] = float(z.sum()) == 2048.0
            done.set()
            comm.close()
        else:
            done.wait(120)  # stays out of step 2, holds no collective in flight
            comm.abort()
    except Exception as e:
        out["error"] = repr(e)
        done.set()
    finally:
        tdist.destroy_process_group()
    q.put((rank, out))


def test_rank_that_stops_calling_is_detected_by_the_deadline():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, done)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert "error" not in res[0] and "error" not in res[1], res
    r0 = res[0]
    assert r0["step1"] and res[1]["step1"]
    assert "timed out" in r0["step2"] and "aborted" in r0["step2"], r0
    assert 2.5 < r0["seconds"] < 30, r0
    assert "aborted" in r0["after"], r0
    assert r0["gpu_ok"]
