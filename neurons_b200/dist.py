"""Multi-GPU sharding of the quantized-matmul path (libnq_dist.so, NCCL).

One process per GPU.  torch.distributed is only used to hand the NCCL
communicator id from rank 0 to the other ranks; the collectives themselves
run inside libnq_dist.so on the caller's stream:

    comm = Comm()                                    # after init_process_group
    row0, rows = tp_shard(N, comm.size, comm.rank)   # this rank's weight rows
    y = tp_quantized_matmul(comm, x, wq[row0:row0+rows], s[...], b[...], N)
    y_mine = ep_moe_switch(comm, x_mine, T, idx_mine, sc_mine, gate, up, down, E)

The reference runs on a single device and has no counterpart of these calls;
they shard mlx_ops::lin (compute/src/compute/model/mlx_ops.h:28-42) by weight
rows and the MoE switch step
(compute/src/compute/model/qwen3_transformer_moe_model_mlx.cpp:29-79) by
experts and tokens.
"""
import ctypes
import os

import torch

from . import ops
from ._lib import NQError, lib as _nq_lib

_HERE = os.path.dirname(os.path.abspath(__file__))
DIST_LIB_PATH = os.path.join(_HERE, "libnq_dist.so")
NQ_COMM_ID_BYTES = 128

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
U64 = ctypes.c_size_t
PI64 = ctypes.POINTER(ctypes.c_int64)

SIGNATURES = {
    "nq_dist_last_error": (ctypes.c_char_p, []),
    "nq_comm_unique_id": (I, [P]),
    "nq_comm_init": (I, [ctypes.POINTER(P), I, I, P]),
    "nq_comm_destroy": (I, [P]),
    "nq_comm_abort": (I, [P]),
    "nq_comm_rank": (I, [P]),
    "nq_comm_size": (I, [P]),
    "nq_comm_symmetric_alloc": (I, [P, U64]),
    "nq_comm_symmetric_ptr": (P, [P, U64]),
    "nq_comm_take_error": (I, [P, ctypes.POINTER(ctypes.c_uint)]),
    "nq_comm_wait": (I, [P, P, I64]),
    "nq_comm_set_timeout": (I, [P, I64]),
    "nq_tp_quantized_matmul_fused": (I, [P, P, I64, P, P, P, I64, I64, I, I, P, P]),
    "nq_tp_shard": (I, [I64, I, I, PI64, PI64]),
    "nq_ep_shard": (I, [I64, I, I, PI64, PI64]),
    "nq_ep_token_shard": (I, [I64, I, I, PI64, PI64]),
    "nq_tp_workspace_size": (U64, [I64, I64, I]),
    "nq_ep_workspace_size": (U64, [I64, I64, I64, I64, I64, I]),
    "nq_tp_quantized_matmul": (I, [P, P, I64, P, P, P, I64, I64, I, I, P, P, U64, P]),
    "nq_ep_moe_switch": (I, [P, P, I64, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P, P, I,
                             I, P, U64, P, P]),
    "nq_ep_fused_arena_size": (U64, [I64, I64, I64, I]),
    "nq_ep_fused_workspace_size": (U64, [I64, I64, I64, I64, I64, I]),
    "nq_ep_moe_switch_fused": (I, [P, P, I64, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P, P,
                                   I, I, U64, P, U64, P, P]),
}

_dist_lib = None


def dist_lib():
    """libnq_dist.so with its signatures (loads libnq.so first)."""
    global _dist_lib
    if _dist_lib is None:
        _nq_lib()
        if not os.path.exists(DIST_LIB_PATH):
            raise ImportError(f"neurons_b200: {DIST_LIB_PATH} is missing -- build it with "
                              "`python -m neurons_b200.build`")
        h = ctypes.CDLL(DIST_LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _dist_lib = h
    return _dist_lib


def _check(status):
    if status != 0:
        msg = dist_lib().nq_dist_last_error()
        raise NQError(status, msg.decode() if msg else "")


def _split(fn, n, nranks, rank):
    a, b = ctypes.c_int64(0), ctypes.c_int64(0)
    _check(getattr(dist_lib(), fn)(n, nranks, rank, ctypes.byref(a), ctypes.byref(b)))
    return a.value, b.value


def tp_shard(N, nranks, rank):
    """(first row, rows) of the weight rows rank `rank` holds; N % nranks == 0."""
    return _split("nq_tp_shard", N, nranks, rank)


def ep_shard(E, nranks, rank):
    """(first expert, experts) rank `rank` holds; E % nranks == 0."""
    return _split("nq_ep_shard", E, nranks, rank)


def ep_token_shard(T, nranks, rank):
    """(first token, tokens) rank `rank` owns; T % nranks == 0."""
    return _split("nq_ep_token_shard", T, nranks, rank)


def tp_workspace_size(M, N, nranks):
    return int(dist_lib().nq_tp_workspace_size(M, N, nranks))


def ep_workspace_size(T, E, top_k, H, I_, nranks):
    return int(dist_lib().nq_ep_workspace_size(T, E, top_k, H, I_, nranks))


def ep_fused_arena_size(T, top_k, H, nranks):
    return int(dist_lib().nq_ep_fused_arena_size(T, top_k, H, nranks))


def ep_fused_workspace_size(T, E, top_k, H, I_, nranks):
    return int(dist_lib().nq_ep_fused_workspace_size(T, E, top_k, H, I_, nranks))


class Comm:
    """An NCCL communicator over the ranks of a torch.distributed group, on the
    current CUDA device.  Rank 0 makes the id; torch.distributed broadcasts it."""

    def __init__(self, group=None):
        import torch.distributed as tdist
        ident = ctypes.create_string_buffer(NQ_COMM_ID_BYTES)
        if not tdist.is_initialized():  # a single process: a communicator of one rank
            self.rank, self.size = 0, 1
            _check(dist_lib().nq_comm_unique_id(ident))
        else:
            self.rank = tdist.get_rank(group)
            self.size = tdist.get_world_size(group)
            if self.rank == 0:
                _check(dist_lib().nq_comm_unique_id(ident))
            box = [bytes(ident.raw) if self.rank == 0 else None]
            tdist.broadcast_object_list(box, src=tdist.get_global_rank(group, 0) if group else 0,
                                        group=group)
            ident = ctypes.create_string_buffer(box[0], NQ_COMM_ID_BYTES)
        self.handle = P()
        self.arena_bytes = 0
        _check(dist_lib().nq_comm_init(ctypes.byref(self.handle), self.size, self.rank, ident))

    def symmetric_alloc(self, nbytes):
        """Collective: allocate the symmetric arena (same size on every rank)."""
        _check(dist_lib().nq_comm_symmetric_alloc(self.handle, nbytes))
        self.arena_bytes = nbytes

    def symmetric_tensor(self, offset, shape, dtype=torch.bfloat16):
        """A torch view of the arena at a byte offset (the same buffer on every rank)."""
        n = 1
        for d in shape:
            n *= d
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        if offset % 256 or offset + nbytes > self.arena_bytes:
            raise NQError(1, "symmetric_tensor: outside the arena or not 256-byte aligned")
        ptr = dist_lib().nq_comm_symmetric_ptr(self.handle, offset)
        if not ptr:
            raise NQError(1, "symmetric_tensor: no arena")
        return _wrap_device(ptr, shape, dtype)

    def take_error(self):
        v = ctypes.c_uint(0)
        _check(dist_lib().nq_comm_take_error(self.handle, ctypes.byref(v)))
        return v.value

    def wait(self, timeout_ms, stream=None):
        """Bounded wait for the work enqueued on the stream (default: the
        current one): raises NQError (ComputeError) and aborts the
        communicator when NCCL reports an error or the deadline passes."""
        st = P(stream.cuda_stream) if stream is not None else ops._stream()
        _check(dist_lib().nq_comm_wait(self.handle, st, timeout_ms))

    def set_timeout(self, timeout_ms):
        """timeout_ms > 0: every sharded call ends with wait(timeout_ms)."""
        _check(dist_lib().nq_comm_set_timeout(self.handle, timeout_ms))

    def close(self):
        if self.handle:
            _check(dist_lib().nq_comm_destroy(self.handle))
            self.handle = P()

    def abort(self):
        if self.handle:
            _check(dist_lib().nq_comm_abort(self.handle))
            self.handle = P()


def _ptr(t):
    return P(t.data_ptr()) if t is not None else None


def _wrap_device(ptr, shape, dtype):
    """A torch tensor over device memory owned by the library (no copy)."""
    import numpy as np  # noqa: F401  (dtype sizes only)
    n = 1
    for d in shape:
        n *= d
    nbytes = n * torch.empty(0, dtype=dtype).element_size()
    dev = torch.cuda.current_device()

    class _Mem:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                    "version": 3, "strides": None}
    t = torch.as_tensor(_Mem(), device=f"cuda:{dev}")
    return t.view(dtype).view(shape)


def tp_quantized_matmul_fused(comm, x, wq_shard, s_shard, b_shard, N, out, group_size=64, bits=4):
    """tp_quantized_matmul with the all-gather fused into the kernel's stores:
    `out` ([M, N] bf16) must be a symmetric_tensor of the communicator."""
    ops._need(x, "x", (torch.bfloat16,))
    ops._need(wq_shard, "w", ops._PACKED)
    K = int(x.shape[-1])
    M = x.numel() // K
    _check(dist_lib().nq_tp_quantized_matmul_fused(
        comm.handle, _ptr(x), M, _ptr(wq_shard), _ptr(s_shard), _ptr(b_shard), N, K, bits,
        group_size, _ptr(out), ops._stream()))
    return out


def tp_quantized_matmul(comm, x, wq_shard, s_shard, b_shard, N, group_size=64, bits=4, out=None,
                        workspace=None):
    """y [M, N] = x . W^T with this rank holding rows tp_shard(N, ...) of W."""
    ops._need(x, "x", (torch.bfloat16,))
    ops._need(wq_shard, "w", ops._PACKED)
    K = int(x.shape[-1])
    M = x.numel() // K
    if out is None:
        out = torch.empty(tuple(x.shape[:-1]) + (N,), dtype=torch.bfloat16, device=x.device)
    need = tp_workspace_size(M, N, comm.size)
    if workspace is None and need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    _check(dist_lib().nq_tp_quantized_matmul(
        comm.handle, _ptr(x), M, _ptr(wq_shard), _ptr(s_shard), _ptr(b_shard), N, K, bits,
        group_size, _ptr(out), _ptr(workspace), workspace.numel() if workspace is not None else 0,
        ops._stream()))
    return out


def ep_moe_switch(comm, x_shard, T, idx_shard, scores_shard, gate, up, down, E, group_size=64,
                  bits=4, workspace=None, out=None):
    """This rank's tokens' switch-step outputs [T/P, H], experts sharded over
    the ranks (gate/up/down: this rank's experts, (wq, scales, biases))."""
    ops._need(x_shard, "x", (torch.bfloat16,))
    H = int(x_shard.shape[1])
    top_k = int(idx_shard.shape[1])
    I_ = int(gate[0].shape[1])
    need = ep_workspace_size(T, E, top_k, H, I_, comm.size)
    if need == 0:
        raise NQError(1, "ep_moe_switch: T and E must be multiples of the number of ranks")
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=x_shard.device)
    if out is None:
        out = torch.empty_like(x_shard)
    _check(dist_lib().nq_ep_moe_switch(
        comm.handle, _ptr(x_shard), T, H, I_, E, top_k, _ptr(idx_shard), _ptr(scores_shard),
        _ptr(gate[0]), _ptr(gate[1]), _ptr(gate[2]), _ptr(up[0]), _ptr(up[1]), _ptr(up[2]),
        _ptr(down[0]), _ptr(down[1]), _ptr(down[2]), bits, group_size, _ptr(workspace),
        workspace.numel(), _ptr(out), ops._stream()))
    return out


def ep_moe_switch_fused(comm, x_shard, T, idx_shard, scores_shard, gate, up, down, E,
                        arena_offset, group_size=64, bits=4, workspace=None, out=None):
    """ep_moe_switch with the token dispatch and the combine as an all-to-all
    over NVLink (peer stores into the symmetric arena region at arena_offset,
    ep_fused_arena_size bytes) instead of NCCL collectives."""
    ops._need(x_shard, "x", (torch.bfloat16,))
    H = int(x_shard.shape[1])
    top_k = int(idx_shard.shape[1])
    I_ = int(gate[0].shape[1])
    need = ep_fused_workspace_size(T, E, top_k, H, I_, comm.size)
    if need == 0:
        raise NQError(1, "ep_moe_switch_fused: T and E must be multiples of the number of ranks")
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=x_shard.device)
    if out is None:
        out = torch.empty_like(x_shard)
    _check(dist_lib().nq_ep_moe_switch_fused(
        comm.handle, _ptr(x_shard), T, H, I_, E, top_k, _ptr(idx_shard), _ptr(scores_shard),
        _ptr(gate[0]), _ptr(gate[1]), _ptr(gate[2]), _ptr(up[0]), _ptr(up[1]), _ptr(up[2]),
        _ptr(down[0]), _ptr(down[1]), _ptr(down[2]), bits, group_size, arena_offset,
        _ptr(workspace), workspace.numel(), _ptr(out), ops._stream()))
    return out
