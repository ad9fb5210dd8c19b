"""CPU tests of the multi-GPU layer (libnq_dist.so, include/nq_dist.h):
the library exports what the header declares, the shard plans, and the
tensor- and expert-parallel data flows run as two gloo ranks on the CPU with
the oracle doing the arithmetic -- the same shard bounds (taken from the
library's own plan functions), the same all-gather layouts and the same
reduction of partial sums as the NCCL path, checked against the single-device
oracle result."""
import ctypes
import os
import re
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nq_dist.h")


def declared():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    return sorted(set(re.findall(r"\b(nq_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def dlib(nqlib):
    from neurons_b200 import build
    build.build_dist()
    from neurons_b200.dist import dist_lib
    return dist_lib()


def test_dist_library_exports_every_declared_symbol(dlib):
    for name in declared():
        assert hasattr(dlib, name), name


def test_dist_signatures_cover_header():
    from neurons_b200.dist import SIGNATURES
    assert sorted(SIGNATURES) == declared()


def test_shard_plans(dlib):
    from neurons_b200 import dist
    assert [dist.tp_shard(14336, 8, r) for r in (0, 3, 7)] == [(0, 1792), (5376, 1792),
                                                              (12544, 1792)]
    assert dist.ep_shard(128, 8, 5) == (80, 16)
    assert dist.ep_token_shard(2048, 8, 1) == (256, 256)
    # the shards tile the range exactly
    for n, p in ((4096, 2), (4096, 4), (128256, 8), (96, 3)):
        cover = sorted(dist.tp_shard(n, p, r) for r in range(p))
        assert cover[0][0] == 0 and all(a[0] + a[1] == b[0] for a, b in zip(cover, cover[1:]))
        assert cover[-1][0] + cover[-1][1] == n


@pytest.mark.parametrize("n,p,r", [(100, 8, 0), (96, 0, 0), (96, 4, 4), (96, 4, -1), (0, 2, 0)])
def test_shard_plans_reject(dlib, n, p, r):
    from neurons_b200 import dist
    from neurons_b200 import NQError
    with pytest.raises(NQError) as e:
        dist.tp_shard(n, p, r)
    assert e.value.code == "InvalidInput"


def test_workspace_sizes(dlib):
    from neurons_b200 import dist
    assert dist.tp_workspace_size(1, 4096, 8) == 0
    assert dist.tp_workspace_size(64, 4096, 2) == 64 * 4096 * 2
    assert dist.ep_workspace_size(2048, 128, 8, 2048, 768, 8) > 2048 * 2048 * 6
    assert dist.ep_workspace_size(2047, 128, 8, 2048, 768, 8) == 0  # T not divisible


def test_failure_detection_arguments(dlib):
    """nq_comm_wait needs a communicator and a positive deadline;
    nq_comm_set_timeout rejects a negative one (no device is touched)."""
    assert dlib.nq_comm_wait(None, None, 1000) == 1
    assert b"nq_comm_wait" in dlib.nq_dist_last_error()
    assert dlib.nq_comm_set_timeout(None, 10) == 1


def test_sharded_calls_validate_before_touching_a_device(dlib):
    dummy = ctypes.c_void_p(16)
    rc = dlib.nq_tp_quantized_matmul(None, dummy, 1, dummy, dummy, dummy, 64, 64, 4, 64, dummy,
                                     None, 0, None)
    assert rc == 1 and b"communicator" in dlib.nq_dist_last_error()


# ------------------------------------------------------------ two gloo ranks

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(fn, *args):
    import torch.multiprocessing as mp
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, fn, args, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        r, res = q.get(timeout=240)
        out[r] = res
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def _rank_main(rank, world, port, fn, args, q):
    import sys
    import datetime
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch.distributed as tdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world,
                             timeout=datetime.timedelta(seconds=120))
    try:
        q.put((rank, globals()[fn](rank, world, *args)))
    except Exception as e:  # report, then exit cleanly so the parent sees it
        q.put((rank, repr(e)))
    finally:
        tdist.destroy_process_group()


def _tp_rank(rank, world, M, N, K, bits, gs):
    import torch
    import torch.distributed as tdist
    from oracle import oracle as O
    from neurons_b200 import dist
    rng = np.random.default_rng(7)
    wq, s, b = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), bits, gs, 0)
    x = O.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    row0, rows = dist.tp_shard(N, world, rank)
    mine = O.qmm(x, wq[row0:row0 + rows], s[row0:row0 + rows], b[row0:row0 + rows], bits, gs)
    # (gloo moves no 16-bit integers: the bf16 bit patterns travel as int32)
    parts = [torch.empty((M, rows), dtype=torch.int32) for _ in range(world)]
    tdist.all_gather(parts, torch.from_numpy(mine.astype(np.int32)))
    g = np.stack([p.numpy().astype(np.uint16) for p in parts])  # [P][M][rows], rank-major
    y = np.empty((M, N), np.uint16)
    for p in range(world):  # the library's rank-major -> row-major step
        y[:, p * rows:(p + 1) * rows] = g[p]
    full = O.qmm(x, wq, s, b, bits, gs)
    return bool(np.array_equal(y, full))


@pytest.mark.parametrize("M,N,K,bits,gs", [(1, 96, 128, 4, 32), (5, 64, 256, 8, 64)])
def test_tensor_parallel_plan_two_gloo_ranks(dlib, M, N, K, bits, gs):
    out = _run_ranks("_tp_rank", M, N, K, bits, gs)
    assert out == {0: True, 1: True}, out


def _ep_rank(rank, world, T, E, k, H, I):
    import torch
    import torch.distributed as tdist
    from oracle import oracle as O
    from neurons_b200 import dist
    rng = np.random.default_rng(11)

    def experts(rows, cols):
        wq, s, b = O.quantize((rng.standard_normal((E * rows, cols)) * 0.02).astype(np.float32),
                              4, 32, 0)
        return wq.reshape(E, rows, -1), s.reshape(E, rows, -1), b.reshape(E, rows, -1)

    gate, up, down = experts(I, H), experts(I, H), experts(H, I)
    x = O.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    idx, sc = O.moe_route(O.f32_to_bf16(rng.standard_normal((T, E)).astype(np.float32)), k)
    t0, nt = dist.ep_token_shard(T, world, rank)
    e0, ne = dist.ep_shard(E, world, rank)
    # dispatch: all-gather this rank's tokens and their routing
    def gather(a, dtype):
        parts = [torch.empty((nt,) + a.shape[1:], dtype=dtype) for _ in range(world)]
        tdist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(a[t0:t0 + nt])))
        return np.concatenate([p.numpy() for p in parts])
    x_all = gather(x.astype(np.int32), torch.int32).astype(np.uint16)
    idx_all = gather(idx, torch.int32)
    sc_all = gather(sc, torch.float32)
    assert np.array_equal(x_all, x) and np.array_equal(idx_all, idx)
    # this rank's experts over all tokens: the slots routed elsewhere weigh 0
    local = (idx_all >= e0) & (idx_all < e0 + ne)
    h = O.moe_hidden(x_all, idx_all, gate, up, 4, 32, rounding=1)
    part = O.bf16_to_f32(O.moe_combine(h, idx_all, np.where(local, sc_all, 0).astype(np.float32),
                                       down, 4, 32, rounding=1))
    # combine: sum the partials, keep this rank's tokens
    tot = torch.from_numpy(part.astype(np.float32))
    tdist.all_reduce(tot)
    mine = tot.numpy()[t0:t0 + nt]
    ref = O.bf16_to_f32(O.moe_switch(x, idx, sc, gate, up, down, 4, 32, rounding=1))[t0:t0 + nt]
    return float(np.linalg.norm(mine - ref) / np.linalg.norm(ref))


def test_expert_parallel_plan_two_gloo_ranks(dlib):
    out = _run_ranks("_ep_rank", 6, 8, 2, 64, 32)
    assert set(out) == {0, 1}
    for r, err in out.items():
        assert isinstance(err, float), err
        assert err < 1e-2, (r, err)


def _ep_a2a_rank(rank, world, T, E, k, H, I):
    """The data flow of nq_ep_moe_switch_fused with the oracle doing the
    arithmetic: each token goes once to every rank holding one of its experts
    (rows of region `rank` of that rank's receive buffer, padding rows routed
    to an expert of another rank with score 0), each rank computes its
    experts' partial sums over the rows it received and returns them to the
    owners, and each owner sums them in rank order."""
    import torch
    import torch.distributed as tdist
    from oracle import oracle as O
    from neurons_b200 import dist
    rng = np.random.default_rng(23)

    def experts(rows, cols):
        wq, s, b = O.quantize((rng.standard_normal((E * rows, cols)) * 0.02).astype(np.float32),
                              4, 32, 0)
        return wq.reshape(E, rows, -1), s.reshape(E, rows, -1), b.reshape(E, rows, -1)

    gate, up, down = experts(I, H), experts(I, H), experts(H, I)
    x = O.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    idx, sc = O.moe_route(O.f32_to_bf16(rng.standard_normal((T, E)).astype(np.float32)), k)
    t0, cap = dist.ep_token_shard(T, world, rank)
    e0, ne = dist.ep_shard(E, world, rank)
    # dispatch plan: pos[t][d] = row of token t in rank d's region for this rank
    pos = -np.ones((cap, world), np.int64)
    cnt = np.zeros(world, np.int64)
    send_x = np.zeros((world, cap, H), np.int32)
    send_idx = np.zeros((world, cap, k), np.int32)
    send_sc = np.zeros((world, cap, k), np.float32)
    for t in range(cap):
        for d in sorted({int(e) // ne for e in idx[t0 + t]}):
            pos[t, d] = cnt[d]
            send_x[d, cnt[d]] = x[t0 + t]
            send_idx[d, cnt[d]] = idx[t0 + t]
            send_sc[d, cnt[d]] = sc[t0 + t]
            cnt[d] += 1

    def exchange(a, dtype):
        """a [P][...] on every rank -> b [P][...] with b[q] = rank q's a[rank]."""
        parts = [torch.empty(a.shape, dtype=dtype) for _ in range(world)]
        tdist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(a)))
        return np.stack([p.numpy()[rank] for p in parts])

    recv_x = exchange(send_x, torch.int32).astype(np.uint16).reshape(world * cap, H)
    recv_idx = exchange(send_idx, torch.int32).reshape(world * cap, k)
    recv_sc = exchange(send_sc, torch.float32).reshape(world * cap, k)
    recv_cnt = exchange(cnt[:, None].astype(np.int32), torch.int32)[:, 0]
    e_pad = (e0 + ne) % E
    for q in range(world):
        recv_idx[q * cap + recv_cnt[q]:(q + 1) * cap] = e_pad
        recv_sc[q * cap + recv_cnt[q]:(q + 1) * cap] = 0
    # this rank's experts over the received rows
    local = (recv_idx >= e0) & (recv_idx < e0 + ne)
    h = O.moe_hidden(recv_x, recv_idx, gate, up, 4, 32, rounding=1)
    part = O.bf16_to_f32(O.moe_combine(h, recv_idx, np.where(local, recv_sc, 0).astype(np.float32),
                                       down, 4, 32, rounding=1)).astype(np.float32)
    # combine: region q of the partials goes back to rank q; sum in rank order
    back = exchange(part.reshape(world, cap, H), torch.float32)  # back[d] = rank d's rows for us
    y = np.zeros((cap, H), np.float32)
    for d in range(world):
        for t in range(cap):
            if pos[t, d] >= 0:
                y[t] += back[d, pos[t, d]]
    ref = O.bf16_to_f32(O.moe_switch(x, idx, sc, gate, up, down, 4, 32, rounding=1))[t0:t0 + cap]
    size_ok = dist.ep_fused_arena_size(T, k, H, world) >= world * cap * H * 6
    return float(np.linalg.norm(y - ref) / np.linalg.norm(ref)) if size_ok else "arena size"


def test_expert_parallel_all_to_all_plan_two_gloo_ranks(dlib):
    out = _run_ranks("_ep_a2a_rank", 6, 8, 2, 64, 32)
    assert set(out) == {0, 1}
    for r, err in out.items():
        assert isinstance(err, float), err
        assert err < 1e-2, (r, err)
