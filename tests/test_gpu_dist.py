"""Two ranks over NCCL (one process per GPU): the tensor-parallel linear and
the expert-parallel switch step (NCCL collectives, and the all-to-all over
peer memory) through libnq_dist.so's C ABI, against the single-GPU calls on
the same seeded inputs.  Needs two GPUs; skipped with one."""
import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


def _worker(rank, world, port, q):
    import sys
    import datetime
    sys.path.insert(0, ROOT)
    import torch.distributed as tdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    tdist.init_process_group("nccl", rank=rank, world_size=world,
                             timeout=datetime.timedelta(seconds=120),
                             device_id=torch.device("cuda", rank))
    out = {}
    try:
        import neurons_b200 as nb
        from neurons_b200 import dist
        comm = dist.Comm()
        comm.symmetric_alloc(8 << 20)
        g = torch.Generator(device="cuda").manual_seed(0)
        for (M, N, K, bits) in ((1, 4096, 4096, 4), (7, 2048, 1024, 8), (300, 2048, 1024, 4)):
            w = torch.randn(N, K, device="cuda", generator=g) * 0.02
            x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
            wq, s, b = nb.quantize(w, 64, bits)
            ref = nb.quantized_matmul(x, wq, s, b, True, 64, bits)
            r0, rows = dist.tp_shard(N, world, rank)
            y = dist.tp_quantized_matmul(comm, x, wq[r0:r0 + rows], s[r0:r0 + rows],
                                         b[r0:r0 + rows], N, 64, bits)
            # this rank's columns are exactly the single-GPU call on its shard
            # (the full-width call may plan its K split differently)
            mine = nb.quantized_matmul(x, wq[r0:r0 + rows], s[r0:r0 + rows], b[r0:r0 + rows],
                                       True, 64, bits)
            torch.cuda.synchronize()
            out[f"tp{M}"] = (_rel(y, ref), torch.equal(y[:, r0:r0 + rows], mine))
            # the fused variant: every rank's columns pushed over NVLink; three
            # calls on the same symmetric buffer (epochs, buffer reuse)
            yf = comm.symmetric_tensor(0, (M, N))
            for _ in range(3):
                yf.zero_()
                dist.tp_quantized_matmul_fused(comm, x, wq[r0:r0 + rows], s[r0:r0 + rows],
                                               b[r0:r0 + rows], N, yf, 64, bits)
            torch.cuda.synchronize()
            out[f"fused{M}"] = (_rel(yf, ref), torch.equal(yf, y))
        E, k, H, I = 16, 4, 512, 256
        gate, up, down = (nb.quantize(torch.randn(E, n, kk, device="cuda", generator=g) * 0.02)
                          for n, kk in ((I, H), (I, H), (H, I)))
        e0, ne = dist.ep_shard(E, world, rank)
        loc = lambda t: tuple(a[e0:e0 + ne].contiguous() for a in t)
        for T in (64, 512):
            x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
            idx, sc = nb.moe_route(torch.randn(T, E, device="cuda", generator=g)
                                   .to(torch.bfloat16), k)
            ref = nb.moe_switch(x, idx, sc, gate, up, down)
            t0, nt = dist.ep_token_shard(T, world, rank)
            y = dist.ep_moe_switch(comm, x[t0:t0 + nt].contiguous(), T,
                                   idx[t0:t0 + nt].contiguous(), sc[t0:t0 + nt].contiguous(),
                                   loc(gate), loc(up), loc(down), E)
            torch.cuda.synchronize()
            out[f"ep{T}"] = (_rel(y, ref[t0:t0 + nt]), True)
            # the all-to-all over NVLink; three calls on the same arena region
            off = 4 << 20
            assert off + dist.ep_fused_arena_size(T, k, H, world) <= 8 << 20
            for _ in range(3):
                yf = dist.ep_moe_switch_fused(comm, x[t0:t0 + nt].contiguous(), T,
                                              idx[t0:t0 + nt].contiguous(),
                                              sc[t0:t0 + nt].contiguous(), loc(gate), loc(up),
                                              loc(down), E, off)
            torch.cuda.synchronize()
            out[f"epf{T}"] = (_rel(yf, ref[t0:t0 + nt]), float((yf.float() - y.float()).abs().max()))
        out["device_error"] = (float(nb.take_device_error()), True)
        out["comm_error"] = (float(comm.take_error()), True)
        comm.close()
    except Exception as e:
        out["error"] = repr(e)
    finally:
        tdist.destroy_process_group()
    q.put((rank, out))


def test_two_rank_tensor_and_expert_parallel():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r, out in res.items():
        assert "error" not in out, (r, out)
        assert out["device_error"][0] == 0 and out["comm_error"][0] == 0
        for key in ("fused1", "fused7", "fused300"):
            rel, same_as_nccl = out[key]
            assert rel < 1e-2 and same_as_nccl, (r, key, out[key])
        for key in ("tp1", "tp7", "tp300"):
            rel, same_cols = out[key]
            assert rel < 1e-2 and same_cols, (r, key, out[key])
        for key in ("ep64", "ep512", "epf64", "epf512"):
            assert out[key][0] < 1e-2, (r, key, out[key])
