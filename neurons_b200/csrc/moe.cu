// moe.cu -- Qwen3-MoE switch step on B200: router top-k, expert grouping,
// SwiGLU gate/up + down projections through the quantized matmul kernels,
// and the score-weighted combine.
//
// Restates compute/src/compute/model/qwen3_transformer_moe_model_mlx.cpp:29-79
// (router :36-48, gather_qmm :69-74, SwiGLU :71, weighted sum :77-78), batched
// over T tokens instead of the per-token loop at :479-486.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "nq.h"

#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

constexpr int kMaxTopK = 32;

// One warp per token.  Selection compares the logits (softmax is monotonic);
// equal logits prefer the lower expert index; output in descending order.
__global__ void route_kernel(const uint16_t *__restrict__ logits, int64_t T, int E, int top_k,
                             int32_t *__restrict__ idx, float *__restrict__ scores) {
    pdl_launch_dependents();
    pdl_wait();  // the logits come from the previous kernel
    const int lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const uint16_t *l = logits + t * E;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, bf16_to_f32(l[e]));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int e = lane; e < E; e += 32) sum += expf(bf16_to_f32(l[e]) - mx);
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    // experts already selected, as a bitmask over this lane's experts
    // (E <= 1024 -> at most 32 per lane)
    uint32_t taken = 0;
    int sel[kMaxTopK];
    float psel[kMaxTopK];
    float psum = 0.0f;
    for (int j = 0; j < top_k; ++j) {
        float bv = -INFINITY;
        int be = 0x7fffffff;
        for (int i = 0, e = lane; e < E; ++i, e += 32) {
            if (taken & (1u << i)) continue;
            const float v = bf16_to_f32(l[e]);
            if (be == 0x7fffffff || v > bv || (v == bv && e < be)) {
                bv = v;
                be = e;
            }
        }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (oe != 0x7fffffff && (be == 0x7fffffff || ov > bv || (ov == bv && oe < be))) {
                bv = ov;
                be = oe;
            }
        }
        sel[j] = be;
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        psel[j] = expf(bv - mx) / sum;
        psum += psel[j];
    }
    if (lane == 0) {
        for (int j = 0; j < top_k; ++j) {
            idx[t * top_k + j] = sel[j];
            scores[t * top_k + j] = psel[j] / psum;
        }
    }
}

// counts[e - e0] = number of (token, slot) pairs routed to expert e, for the
// experts [e0, e0 + ne) this call serves; indices outside [0, E) raise the
// bad-index bit of the device error word
__global__ void count_kernel(const int32_t *__restrict__ idx, int64_t pairs, int E, int e0, int ne,
                             int32_t *__restrict__ counts, unsigned int *err) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= pairs) return;
    const int e = idx[i];
    if (e < 0 || e >= E) {
        atomicOr(err, kErrBadIndex);
        return;
    }
    const int l = e - e0;
    if (l >= 0 && l < ne) atomicAdd(&counts[l], 1);
}

// exclusive prefix sum over experts (single block, E <= 1024); clears cursors.
// With `tiles`, also lists the tensor-core tiles: expert e's run of grouped
// rows [offsets[e], offsets[e] + counts[e]) cut into pieces of at most
// kMoeTileTokens, as {e, first row, count, 0}; *n_tiles = their number.
__global__ void scan_kernel(const int32_t *__restrict__ counts, int E, int32_t *__restrict__ offsets,
                            int32_t *__restrict__ cursor, int4 *__restrict__ tiles,
                            int32_t *__restrict__ n_tiles) {
    __shared__ int32_t buf[1024];
    const int t = threadIdx.x;
    const int32_t c = t < E ? counts[t] : 0;
    buf[t] = c;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
        const int32_t v = t >= o ? buf[t - o] : 0;
        __syncthreads();
        buf[t] += v;
        __syncthreads();
    }
    const int32_t off = buf[t] - c;
    if (t < E) {
        offsets[t] = off;
        cursor[t] = 0;
    }
    if (tiles == nullptr) return;
    const int32_t nt = (c + kMoeTileTokens - 1) / kMoeTileTokens;
    __syncthreads();
    buf[t] = nt;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
        const int32_t v = t >= o ? buf[t - o] : 0;
        __syncthreads();
        buf[t] += v;
        __syncthreads();
    }
    const int32_t first = buf[t] - nt;
    for (int i = 0; i < nt; ++i)
        tiles[first + i] = make_int4(t, off + i * kMoeTileTokens,
                                     min(kMoeTileTokens, c - i * kMoeTileTokens), 0);
    if (t == 1023) *n_tiles = buf[1023];
}

// place every pair at offsets[e] + rank; the rank order inside an expert does
// not change any result (each output row depends on its own input row only)
__global__ void fill_kernel(const int32_t *__restrict__ idx, int64_t pairs, int top_k, int E, int e0,
                            int ne, const int32_t *__restrict__ offsets, int32_t *__restrict__ cursor,
                            int32_t *__restrict__ pos_token, int32_t *__restrict__ pos_pair) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= pairs) return;
    const int e = idx[i];
    if (e < 0 || e >= E) return;
    const int l = e - e0;
    if (l < 0 || l >= ne) return;
    const int32_t pos = offsets[l] + atomicAdd(&cursor[l], 1);
    pos_token[pos] = (int32_t)(i / top_k);
    pos_pair[pos] = (int32_t)i;
}

// xg[g] = x[pos_token[g]] for the grouped rows g < sum(counts): one warp per
// row, 16-byte copies (H % 8 == 0, 16-byte aligned rows)
__global__ void group_rows_kernel(const uint16_t *__restrict__ x, int64_t H,
                                  const int32_t *__restrict__ pos_token,
                                  const int32_t *__restrict__ offsets,
                                  const int32_t *__restrict__ counts, int E,
                                  uint16_t *__restrict__ xg) {
    const int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (g >= (int64_t)offsets[E - 1] + counts[E - 1]) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (int64_t)pos_token[g] * H);
    uint4 *dst = reinterpret_cast<uint4 *>(xg + g * H);
    for (int64_t i = lane; i < H / 8; i += 32) dst[i] = src[i];
}

// sum_j bf16(score[t, j]) * d[t*k + j, n] over the slots j routed to experts
// [e0, e0 + ne), slot order 0..k-1; y gets it rounded to bf16, or y_partial
// gets the fp32 sum (the share of one expert shard), or -- with ro.n > 0 --
// the fp32 sum goes to rank q's buffer ro.dst[q] at row ro.row0 + i for the
// token t = q * ro.per + i, rows i >= ro.count[q] being skipped (the
// expert-parallel combine, written straight into the token owners' memory)
__global__ void combine_kernel(const float *__restrict__ d, const float *__restrict__ scores,
                               const int32_t *__restrict__ idx, int e0, int ne, int64_t T,
                               int64_t H, int top_k, uint16_t *__restrict__ y,
                               float *__restrict__ y_partial, const MoeRowsOut ro) {
    pdl_launch_dependents();
    pdl_wait();  // d comes from the down projection
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over T * H / 4
    if (i >= T * (H / 4)) return;
    const int64_t t = i / (H / 4);
    const int64_t n = (i % (H / 4)) * 4;
    float *ro_dst = nullptr;
    if (ro.n > 0) {
        const int64_t q = t / ro.per, r = t % ro.per;
        if (r >= ro.count[q]) return;
        ro_dst = ro.dst[q] + (ro.row0 + r) * H + n;
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < top_k; ++j) {
        const int l = idx[t * top_k + j] - e0;
        if (l < 0 || l >= ne) continue;
        const float sc = bf16_to_f32(f32_to_bf16(scores[t * top_k + j]));
        const float4 v = *reinterpret_cast<const float4 *>(d + (t * top_k + j) * H + n);
        acc.x = __fmaf_rn(sc, v.x, acc.x);
        acc.y = __fmaf_rn(sc, v.y, acc.y);
        acc.z = __fmaf_rn(sc, v.z, acc.z);
        acc.w = __fmaf_rn(sc, v.w, acc.w);
    }
    if (ro_dst) {
        *reinterpret_cast<float4 *>(ro_dst) = acc;
        return;
    }
    if (y_partial) {
        *reinterpret_cast<float4 *>(y_partial + t * H + n) = acc;
        return;
    }
    uint2 out;
    out.x = (uint32_t)f32_to_bf16(acc.x) | ((uint32_t)f32_to_bf16(acc.y) << 16);
    out.y = (uint32_t)f32_to_bf16(acc.z) | ((uint32_t)f32_to_bf16(acc.w) << 16);
    *reinterpret_cast<uint2 *>(y + t * H + n) = out;
}

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

bool fused_combine_enabled() {
    const char *v = std::getenv("NQ_MOE_FUSED_COMBINE");
    return v && v[0] == '1';
}

// Launch as a programmatic dependent of the previous kernel on the stream:
// the kernel may start early and waits (griddepcontrol.wait) before it reads
// what that kernel produced.
template <typename... Args>
cudaError_t launch_pdl(void (*kern)(Args...), unsigned blocks, unsigned threads,
                       cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(threads);
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Workspace layout (each region 256-byte aligned), P = T * top_k pairs:
//   counts[E], offsets[E], cursor[E], pos_token[P], pos_pair[P]   int32
//   tiles[max_tiles] int4, n_tiles int32   (tensor-core tile list)
//   h[P, I]  bf16      (SwiGLU activations, grouped or pair order)
//   d[P, H]  fp32      (down-projection sums, pair order)
//   xg[P, H] bf16      (tokens in grouped order; only when P >= 8 E, the
//                       tensor-core path)
int64_t max_moe_tiles(int64_t P, int64_t E) {
    return (P + kMoeTileTokens - 1) / kMoeTileTokens + std::min<int64_t>(E, P);
}

struct MoeWorkspace {
    int32_t *counts, *offsets, *cursor, *pos_token, *pos_pair;
    int4 *tiles;
    int32_t *n_tiles;
    uint16_t *h;
    float *d;
    uint16_t *xg;
    int32_t *arrivals;  // [T, ceil(H/128)]: the tensor-core down kernel's fused combine
    size_t bytes;
};

// The grouped tensor-core path is taken from 8 pairs per expert on (measured
// at the Qwen3-30B-A3B dims: the grouped GEMV wins at 4 per expert, 187 vs
// 310 us at T = 64; the tensor cores at 8, 318 vs 403 us at T = 128).
inline bool tc_pairs(int64_t P, int64_t E) { return P >= 8 * E; }

// E: experts this call serves (sizes the per-expert arrays); E_total: experts
// the router chose from (decides whether the tensor-core path, and xg, is used)
MoeWorkspace carve(void *base, int64_t T, int64_t E, int64_t top_k, int64_t H, int64_t I,
                   int64_t E_total) {
    MoeWorkspace w;
    const int64_t P = T * top_k;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = static_cast<char *>(base) + off;
        off += align256(bytes);
        return p;
    };
    w.counts = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * E));
    w.offsets = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * E));
    w.cursor = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * E));
    w.pos_token = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * P));
    w.pos_pair = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * P));
    w.tiles = reinterpret_cast<int4 *>(take(sizeof(int4) * max_moe_tiles(P, E)));
    w.n_tiles = reinterpret_cast<int32_t *>(take(sizeof(int32_t)));
    w.h = reinterpret_cast<uint16_t *>(take(sizeof(uint16_t) * P * I));
    w.d = reinterpret_cast<float *>(take(sizeof(float) * P * H));
    w.xg = tc_pairs(P, E_total) ? reinterpret_cast<uint16_t *>(take(sizeof(uint16_t) * P * H))
                                : nullptr;
    w.arrivals = tc_pairs(P, E_total)
                     ? reinterpret_cast<int32_t *>(take(sizeof(int32_t) * T * ((H + 127) / 128)))
                     : nullptr;
    w.bytes = off;
    return w;
}

}  // namespace

cudaError_t launch_moe_route(const uint16_t *logits, int64_t T, int64_t E, int64_t top_k,
                             int32_t *idx, float *scores, cudaStream_t stream) {
    if (T == 0) return cudaSuccess;
    const int warps = 8;
    return launch_pdl(route_kernel, (unsigned)((T + warps - 1) / warps), warps * 32, stream, logits,
                      T, (int)E, (int)top_k, idx, scores);
}

size_t moe_workspace_bytes(int64_t T, int64_t E, int64_t top_k, int64_t H, int64_t I) {
    return carve(nullptr, T, E, top_k, H, I, E).bytes;
}

size_t moe_partial_workspace_bytes(int64_t T, int64_t E, int64_t ne, int64_t top_k, int64_t H,
                                   int64_t I) {
    return carve(nullptr, T, ne, top_k, H, I, E).bytes;
}

// Pairs routed to one expert are processed together ("grouped" mode) once
// there are more pairs than experts; below that every pair is its own
// problem ("pair" mode: no grouping kernels, one weight stream per pair).
// The switch step for the experts [e0, e0 + ne) of E: the weights passed are
// those ne experts.  Serving all experts (e0 = 0, ne = E) writes the bf16
// result to y; serving a shard writes the fp32 partial sum to y_partial.
cudaError_t launch_moe_switch(const uint16_t *x, int64_t T, int64_t H, int64_t I, int64_t E_total,
                              int64_t top_k, const int32_t *idx, const float *scores, int64_t e0,
                              int64_t E, const uint32_t *gw, const uint16_t *gs_,
                              const uint16_t *gb, const uint32_t *uw, const uint16_t *us,
                              const uint16_t *ub, const uint32_t *dw, const uint16_t *ds,
                              const uint16_t *db, int bits, int gsz, void *workspace, uint16_t *y,
                              float *y_partial, cudaStream_t stream, const MoeRowsOut *rows_out) {
    if (T == 0) return cudaSuccess;
    const MoeRowsOut ro = rows_out ? *rows_out : MoeRowsOut{};
    const int64_t P = T * top_k;
    MoeWorkspace ws = carve(workspace, T, E, top_k, H, I, E_total);
    unsigned int *err = device_error_word();
    const int thr = 256;
    const unsigned pblocks = (unsigned)((P + thr - 1) / thr);
    // a shard always groups (pairs of other shards are skipped while grouping)
    const bool grouped = P > E || y_partial != nullptr || ro.n > 0;
    // Tensor-core path once experts average >= 8 tokens (tc_pairs); below
    // that the grouped GEMV streams each expert's weights once.
    const bool use_tc =
        grouped && tc_pairs(P, E_total) && tc_moe_supported(bits, gsz, H, I, E, x, H);
    const int64_t n4 = T * (H / 4);
    const unsigned cblocks = (unsigned)((n4 + thr - 1) / thr);
    cudaError_t e;

    GemvProblems up;
    up.w = gw; up.s = gs_; up.b = gb;
    up.w2 = uw; up.s2 = us; up.b2 = ub;
    up.N = I; up.K = H; up.bits = bits; up.gs = gsz;
    up.x = x; up.x_ld = H;
    up.E = (int)E;
    up.y = ws.h; up.y_ld = I;
    up.swiglu = 1;

    GemvProblems dn;
    dn.w = dw; dn.s = ds; dn.b = db;
    dn.N = H; dn.K = I; dn.bits = bits; dn.gs = gsz;
    dn.x = ws.h; dn.x_ld = I;
    dn.E = (int)E;
    dn.y = ws.d; dn.y_ld = H;
    dn.out_f32 = 1;

    if (grouped) {
        if ((e = cudaMemsetAsync(ws.counts, 0, sizeof(int32_t) * E, stream)) != cudaSuccess)
            return e;
        if (use_tc && (e = cudaMemsetAsync(ws.arrivals, 0,
                                           sizeof(int32_t) * T * ((H + 127) / 128), stream)) !=
                          cudaSuccess)
            return e;
        count_kernel<<<pblocks, thr, 0, stream>>>(idx, P, (int)E_total, (int)e0, (int)E, ws.counts,
                                                   err);
        scan_kernel<<<1, 1024, 0, stream>>>(ws.counts, (int)E, ws.offsets, ws.cursor,
                                            use_tc ? ws.tiles : nullptr, ws.n_tiles);
        fill_kernel<<<pblocks, thr, 0, stream>>>(idx, P, (int)top_k, (int)E_total, (int)e0, (int)E,
                                                  ws.offsets, ws.cursor, ws.pos_token, ws.pos_pair);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        if (use_tc) {
            group_rows_kernel<<<(unsigned)((P + 7) / 8), 256, 0, stream>>>(
                x, H, ws.pos_token, ws.offsets, ws.counts, (int)E, ws.xg);
            TcMoeArgs a;
            a.up = true;
            a.bits = bits;
            a.gs = gsz;
            a.E = E;
            a.N = I;
            a.K = H;
            a.w1 = gw; a.s1 = gs_; a.b1 = gb;
            a.w2 = uw; a.s2 = us; a.b2 = ub;
            a.x = ws.xg;
            a.x_ld = H;
            a.x_rows_total = P;
            a.tiles = ws.tiles;
            a.n_tiles = ws.n_tiles;
            a.max_tiles = max_moe_tiles(P, E);
            a.y = ws.h;
            a.y_ld = I;
            if ((e = launch_tc_moe(a, stream)) != cudaSuccess) return e;
            TcMoeArgs d = a;
            d.up = false;
            d.N = H;
            d.K = I;
            d.w1 = dw; d.s1 = ds; d.b1 = db;
            d.w2 = nullptr; d.s2 = nullptr; d.b2 = nullptr;
            d.x = ws.h;
            d.x_ld = I;
            d.x_rows_total = P;
            d.rows = ws.pos_pair;
            d.y = ws.d;
            d.y_ld = H;
            // The score-weighted combine can run in the down kernel itself
            // (NQ_MOE_FUSED_COMBINE=1) when every token it must write has a
            // routed pair there: the whole switch step (y) and the
            // expert-parallel rows (ro; a token is sent only where one of its
            // experts lives).  The fp32 partial of a shard (y_partial) keeps
            // the combine kernel, which also writes the zero rows of tokens
            // routed elsewhere.  Off by default: measured at T = 2048 (Qwen3
            // dims) the fused step takes 512 us against 466 us, because each
            // down CTA's arrival count and combine add round trips to its
            // tail and the kernel is not persistent, so the tails of its ~14
            // waves do not overlap.
            const bool fuse = y_partial == nullptr && H % 4 == 0 && fused_combine_enabled();
            if (fuse) {
                d.fuse_cnt = ws.arrivals;
                d.idx = idx;
                d.scores = scores;
                d.top_k = (int)top_k;
                d.e0 = (int)e0;
                d.out = y;
                d.ro = ro;
            }
            if ((e = launch_tc_moe(d, stream)) != cudaSuccess) return e;
            if (fuse) return cudaSuccess;
            return launch_pdl(combine_kernel, cblocks, thr, stream, (const float *)ws.d, scores, idx,
                              (int)e0, (int)E, T, H, (int)top_k, y, y_partial, ro);
        }
        // gate/up: problem = expert, its tokens gathered from x, h rows in grouped order
        up.P = (int)E;
        up.expert_is_p = true;
        up.m_count = ws.counts;
        up.m_offset = ws.offsets;
        up.x_rows = ws.pos_token;
        up.max_m = (int)T;  // an expert sees each token at most once
        // token tile sized for the average expert (P / E); busier experts take
        // more passes over their (then L2-resident) weights
        up.tile_m = (int)std::min<int64_t>(32, std::max<int64_t>(8, 2 * ((P + E - 1) / E)));
        // down: problem = expert, rows of h in grouped order, d rows by pair id
        dn.P = (int)E;
        dn.expert_is_p = true;
        dn.m_count = ws.counts;
        dn.m_offset = ws.offsets;
        dn.x_from_offset = true;
        dn.y_rows = ws.pos_pair;
        dn.max_m = up.max_m;
        dn.tile_m = up.tile_m;
    } else {
        // a few tokens over all experts: two kernels, the down one forming
        // the weighted sum (no d round trip, no combine launch)
        if (y && !y_partial && ro.n == 0 && e0 == 0 && E == E_total &&
            moe_small_supported(T, H, I, E, top_k, bits, x))
            return launch_moe_small(x, T, H, I, E, top_k, idx, scores, gw, gs_, gb, uw, us, ub,
                                    dw, ds, db, gsz, ws.h, y, stream);
        // pair i reads token i / top_k
        up.P = (int)P;
        up.M = 1;
        up.expert = idx;
        up.x_div = (int)top_k;
        up.x_batch = (int)T;
        up.max_m = 1;
        dn.P = (int)P;
        dn.M = 1;
        dn.expert = idx;
        dn.x_batch = (int)P;
        dn.max_m = 1;
    }
    if ((e = launch_gemv(up, stream)) != cudaSuccess) return e;
    if ((e = launch_gemv(dn, stream)) != cudaSuccess) return e;
    return launch_pdl(combine_kernel, cblocks, thr, stream, (const float *)ws.d, scores, idx,
                      (int)e0, (int)E, T, H, (int)top_k, y, y_partial, ro);
}

}  // namespace nq

// ---------------------------------------------------------------------------
// nq_moe_switch_static: the switch step without a caller-provided workspace.
//
// Some callers cannot allocate device memory on their own: a runtime that
// hands the library only the tensors it already owns (a pre-planned memory
// arena, an embedding through an FFI that exposes no allocator), or a caller
// that must not trigger an allocation while it runs.  For them the scratch
// that nq_moe_switch takes as `workspace` lives instead in the array below,
// a fixed-size block in the library's own device memory.  Every device that
// loads the library holds it until the process exits.
//
// The array's name is only meaningful to device code.  In host code it is a
// stand-in symbol, not a device address, so the host looks up the real
// address once per device with cudaGetSymbolAddress (with that device
// current) and passes that address to the kernels.
// ---------------------------------------------------------------------------
namespace nq {
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_moe_scratch[kStaticScratchBytes];

constexpr int kScratchMaxDevices = 64;
void *g_scratch_ptr[kScratchMaxDevices];
std::mutex g_scratch_mu;

// Address of g_moe_scratch on the current device; the first call on a device
// performs the lookup.  Returns the CUDA error of the lookup.
cudaError_t static_scratch(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kScratchMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_moe_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace nq

static int static_fail(int status, const std::string &msg) {
    nq::set_error(msg);
    return status;
}

extern "C" int nq_moe_switch_static(const uint16_t *x, int64_t T, int64_t H, int64_t I,
                                    int64_t E, int64_t top_k, const int32_t *topk_idx,
                                    const float *topk_scores, const uint32_t *gate_w,
                                    const uint16_t *gate_s, const uint16_t *gate_b,
                                    const uint32_t *up_w, const uint16_t *up_s,
                                    const uint16_t *up_b, const uint32_t *down_w,
                                    const uint16_t *down_s, const uint16_t *down_b, int bits,
                                    int group_size, uint16_t *y, void *stream) {
    if (T < 0 || E <= 0 || E > 1024 || top_k <= 0 || top_k > 32 || top_k > E || H <= 0 || I <= 0)
        return static_fail(NQ_INVALID_INPUT,
                           "nq_moe_switch_static: need 0 < top_k <= min(E, 32), E <= 1024, "
                           "H > 0, I > 0");
    const size_t need = nq::moe_workspace_bytes(T, E, top_k, H, I);
    if (need > nq::kStaticScratchBytes)
        return static_fail(NQ_INVALID_INPUT,
                           "nq_moe_switch_static: this call needs " + std::to_string(need) +
                               " bytes of scratch but the library's static scratch holds " +
                               std::to_string(nq::kStaticScratchBytes) +
                               " bytes; pass fewer tokens per call, or use nq_moe_switch "
                               "with a caller-provided workspace");
    if (nq_device_count() == 0)
        return static_fail(NQ_BACKEND_NOT_AVAILABLE, "nq_moe_switch_static: no CUDA device");
    void *scratch = nullptr;
    const cudaError_t e = nq::static_scratch(&scratch);
    if (e != cudaSuccess)
        return static_fail(NQ_COMPUTE_ERROR,
                           std::string("nq_moe_switch_static: cudaGetSymbolAddress failed: ") +
                               cudaGetErrorString(e));
    // The same validation and kernels as nq_moe_switch, on the static block.
    return nq_moe_switch(x, T, H, I, E, top_k, topk_idx, topk_scores, gate_w, gate_s, gate_b,
                         up_w, up_s, up_b, down_w, down_s, down_b, bits, group_size, scratch,
                         nq::kStaticScratchBytes, y, stream);
}
