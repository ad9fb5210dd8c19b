"""Helpers shared by the GPU tests: numpy <-> torch transfers of raw bit
patterns, seeded workloads, and the matmul tolerance of the parity contract."""
import numpy as np
import torch

from oracle import oracle as O

# Matmul parity contract (fp32 accumulation, bf16 out):
#   rel = |y - r| / max(|r|, FLOOR * rms(r));  max(rel) <= MAX_REL, mean(rel) <= MEAN_REL
MAX_REL = 2e-2
MEAN_REL = 2e-3
FLOOR = 1e-3


def rel_errors(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref)) if ref.size else 1.0
    den = np.maximum(np.abs(ref), FLOOR * rms + 1e-30)
    return np.abs(y - ref) / den


def assert_close(y_bits, ref, what=""):
    """y_bits: bf16 bit patterns from the GPU; ref: the oracle's bf16 output (bit
    patterns) -- both sides rounded to bf16 as the contract's "bf16 out" says."""
    y = O.bf16_to_f32(y_bits)
    r = O.bf16_to_f32(ref) if np.asarray(ref).dtype == np.uint16 else np.asarray(ref)
    rel = rel_errors(y, r)
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    assert rel.max() <= MAX_REL, f"{what}: max rel err {rel.max():.3e} > {MAX_REL}"
    assert rel.mean() <= MEAN_REL, f"{what}: mean rel err {rel.mean():.3e} > {MEAN_REL}"
    return rel.max(), rel.mean()


def dev_bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).view(
        torch.bfloat16).cuda()


def dev_u32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).cuda()


def dev_i32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).cuda()


def dev_f32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host_u16(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def host_u32(t):
    return t.detach().contiguous().cpu().view(torch.int32).numpy().view(np.uint32)


def weights(rng, rows, cols, std=0.02):
    return (rng.standard_normal((rows, cols)) * std).astype(np.float32)


def acts(rng, rows, cols):
    return O.f32_to_bf16(rng.standard_normal((rows, cols)).astype(np.float32))


def workspace_hidden(ws, T, E, k, H, I):
    """The SwiGLU activations h the GPU wrote into the caller-owned workspace,
    returned in pair order (t*k + j).  Follows the workspace layout of
    neurons_b200/csrc/moe.cu: counts[E], offsets[E], cursor[E], pos_token[P],
    pos_pair[P] (int32), tiles[ceil(P/256) + min(E, P)] (int4), n_tiles (int32),
    h[P, I] (bf16), d[P, H] (fp32), each region aligned to 256 bytes; h is in
    pair order when P <= E, else grouped by expert with pos_pair giving each
    row's pair."""
    P = T * k
    a = lambda n: (n + 255) // 256 * 256
    raw = ws.cpu().numpy()
    off = 3 * a(4 * E)
    pos_pair = raw[off + a(4 * P): off + a(4 * P) + 4 * P].view(np.int32)
    max_tiles = (P + 255) // 256 + min(E, P)
    hoff = off + 2 * a(4 * P) + a(16 * max_tiles) + a(4)
    h = raw[hoff: hoff + 2 * P * I].view(np.uint16).reshape(P, I)
    if P <= E:
        return h.copy()
    out = np.zeros_like(h)
    out[pos_pair] = h
    return out
