// gemv.cu -- skinny quantized matmul (decode GEMV / small-M GEMM), sm_100a.
//
// y[m, n] = sum_k x[m, k] * w_hat[n, k],  w_hat = bf16(bf16(s*q) + b)
// (the MLX CPU dequantized value, bit for bit), fp32 accumulation.
//
// Work decomposition
//   * A warp owns a 16-row tile of W and a contiguous range of "k-blocks"
//     (16 packed words per row: 128 codes at 4 bits, 64 codes at 8 bits).
//   * Per k-block each lane issues two 128-bit streaming loads (rows g and
//     g+8 of the tile, g = lane/4), i.e. a quad of lanes reads 64 contiguous
//     bytes of a row; the codes are dequantized in registers straight into
//     mma.sync m16n8k16 A fragments (weights are the MMA "M" side, tokens the
//     "N" side, up to 8 tokens per n-tile).  The k order inside a fragment is
//     permuted to (k, k+4) pairs so that a 4-bit word splits into fragments
//     with one lop3 per pair; the activation fragments use the same
//     permutation, so the dot product is unchanged.
//   * The warps of a CTA split K; their partial tiles are summed in shared
//     memory.  When the grid also splits K across CTAs, those CTAs form a
//     thread-block cluster and the partials are summed through distributed
//     shared memory -- no global scratch and no atomics.
//   * Problems (blockIdx.z) cover batched / gathered calls: gather_qmm (one
//     problem per index) and the MoE expert groups (one problem per expert
//     with a device-side token list).
//   * Programmatic dependent launch: weights and scales are fetched before
//     griddepcontrol.wait, so back-to-back projections overlap the weight
//     stream of one with the tail of the previous.
#include <cooperative_groups.h>

#include <algorithm>

#include "nq_common.cuh"
#include "nq_internal.h"

namespace cg = cooperative_groups;

namespace nq {
namespace {

struct GemvParams {
    const uint32_t *w, *w2;
    const uint16_t *s, *b, *s2, *b2;
    int64_t N, K, Kw, G;  // out rows, in features, words per row, groups per row
    int gs_shift;         // log2(group size): group sizes are 32, 64 or 128
    const uint16_t *x;
    int64_t x_ld;
    int P, M, E, x_batch;
    const int32_t *expert, *m_count, *m_offset, *x_rows, *lhs, *y_rows;
    int expert_is_p, x_from_offset;
    void *y;
    int64_t y_ld;
    int out_f32, swiglu;
    int kb_total;
    unsigned int *err;
};

__device__ __forceinline__ uint4 ldg_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ldg16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint2 ldg8(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ldg_u16(const uint16_t *p) {
    uint16_t r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int kUnroll = 2;  // k-blocks whose weight loads are in flight together

// One k-block of one weight matrix against NT token tiles.
//   4 bits: word i of this lane holds codes k0+8i .. k0+8i+7; the two mma
//   steps use pairs (q0,q4),(q1,q5) and (q2,q6),(q3,q7), the activations the
//   same pairs of x.
//   8 bits: word i holds codes k0+4i .. k0+4i+3; one mma step.
template <int BITS, int NT>
__device__ __forceinline__ void kblock_mma(float (&acc)[NT][4], const uint4 &wa, const uint4 &wb,
                                           uint16_t sa, uint16_t ba, uint16_t sb, uint16_t bb,
                                           const uint16_t *const (&xrow)[NT], int64_t kcode0,
                                           bool kvalid) {
    const uint32_t wA[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t wB[4] = {wb.x, wb.y, wb.z, wb.w};
    if constexpr (BITS == 4) {
        const Dq4 da = make_dq4(sa, ba), db = make_dq4(sb, bb);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t a00 = dq4_pair(q4_pair_biased(wA[i], 0), da);
            const uint32_t a01 = dq4_pair(q4_pair_biased(wB[i], 0), db);
            const uint32_t a02 = dq4_pair(q4_pair_biased(wA[i], 1), da);
            const uint32_t a03 = dq4_pair(q4_pair_biased(wB[i], 1), db);
            const uint32_t a10 = dq4_pair(q4_pair_biased(wA[i], 2), da);
            const uint32_t a11 = dq4_pair(q4_pair_biased(wB[i], 2), db);
            const uint32_t a12 = dq4_pair(q4_pair_biased(wA[i], 3), da);
            const uint32_t a13 = dq4_pair(q4_pair_biased(wB[i], 3), db);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                uint4 xv = make_uint4(0, 0, 0, 0);
                if (xrow[nt] != nullptr && kvalid) xv = ldg16(xrow[nt] + kcode0 + 8 * i);
                // (x0,x4) (x1,x5) (x2,x6) (x3,x7)
                const uint32_t b00 = prmt(xv.x, xv.z, 0x5410u), b01 = prmt(xv.x, xv.z, 0x7632u);
                const uint32_t b10 = prmt(xv.y, xv.w, 0x5410u), b11 = prmt(xv.y, xv.w, 0x7632u);
                mma16816(acc[nt], a00, a01, a02, a03, b00, b01);
                mma16816(acc[nt], a10, a11, a12, a13, b10, b11);
            }
        }
    } else {
        const Dq8 da = make_dq8(sa, ba), db = make_dq8(sb, bb);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t a0 = dq8_pair(wA[i], 0, 1, da);
            const uint32_t a1 = dq8_pair(wB[i], 0, 1, db);
            const uint32_t a2 = dq8_pair(wA[i], 2, 3, da);
            const uint32_t a3 = dq8_pair(wB[i], 2, 3, db);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                uint2 xv = make_uint2(0, 0);
                if (xrow[nt] != nullptr && kvalid) xv = ldg8(xrow[nt] + kcode0 + 4 * i);
                mma16816(acc[nt], a0, a1, a2, a3, xv.x, xv.y);
            }
        }
    }
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

template <int BITS, int NT, bool DUAL>
__global__ void __launch_bounds__(256) qgemv_kernel(const GemvParams prm) {
    constexpr int NACC = DUAL ? 2 : 1;
    extern __shared__ float red[];  // [warps][NACC][NT][4][32]

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int p = blockIdx.z;

    pdl_launch_dependents();

    // index arrays may be produced by the previous kernel on the stream
    const bool indexed = prm.expert || prm.m_count || prm.x_rows || prm.lhs || prm.y_rows;
    if (indexed) pdl_wait();

    int e = prm.expert_is_p ? p : (prm.expert ? prm.expert[p] : 0);
    bool bad = false;
    if (e < 0 || e >= prm.E) {
        bad = true;
        e = 0;
    }
    const int Mp = prm.m_count ? prm.m_count[p] : prm.M;
    const int off = prm.m_offset ? prm.m_offset[p] : p * prm.M;
    int xi = prm.lhs ? prm.lhs[p] : (prm.x_batch == prm.P ? p : 0);
    if (xi < 0 || xi >= prm.x_batch) {
        bad = true;
        xi = 0;
    }
    if (bad && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
        atomicOr(prm.err, kErrBadIndex);
    if (Mp <= 0) return;  // uniform over the cluster (same problem)

    const int64_t n0 = (int64_t)blockIdx.x * 16;
    const int64_t ra = n0 + g, rb = n0 + g + 8;
    const bool va = ra < prm.N && !bad, vb = rb < prm.N && !bad;
    const int64_t wrow_a = ((int64_t)e * prm.N + ra) * prm.Kw;
    const int64_t wrow_b = ((int64_t)e * prm.N + rb) * prm.Kw;
    const int64_t srow_a = ((int64_t)e * prm.N + ra) * prm.G;
    const int64_t srow_b = ((int64_t)e * prm.N + rb) * prm.G;

    const int tw = gridDim.y * warps;
    const int gw = blockIdx.y * warps + warp;
    const int kb_lo = (int)(((int64_t)gw * prm.kb_total) / tw);
    const int kb_hi = (int)(((int64_t)(gw + 1) * prm.kb_total) / tw);
    constexpr int kCodesPerWord = 32 / BITS;

    bool waited = indexed;

    for (int m0 = 0; m0 < Mp; m0 += 8 * NT) {
        float acc[NACC][NT][4];
#pragma unroll
        for (int a = 0; a < NACC; ++a)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[a][nt][j] = 0.0f;

        const uint16_t *xrow[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xrow[nt] = nullptr;

        for (int kb0 = kb_lo; kb0 < kb_hi; kb0 += kUnroll) {
            uint4 wa[NACC][kUnroll], wb[NACC][kUnroll];
            uint16_t sa[NACC][kUnroll], ba[NACC][kUnroll], sb[NACC][kUnroll], bb[NACC][kUnroll];
            bool kv[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int kb = kb0 + u;
                const int64_t wbase = (int64_t)kb * 16 + 4 * c;
                kv[u] = kb < kb_hi && wbase < prm.Kw;
                const int64_t grp = (wbase * kCodesPerWord) >> prm.gs_shift;
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    const uint32_t *W = a ? prm.w2 : prm.w;
                    const uint16_t *S = a ? prm.s2 : prm.s;
                    const uint16_t *B = a ? prm.b2 : prm.b;
                    wa[a][u] = make_uint4(0, 0, 0, 0);
                    wb[a][u] = make_uint4(0, 0, 0, 0);
                    sa[a][u] = ba[a][u] = sb[a][u] = bb[a][u] = 0;
                    if (kv[u] && va) {
                        wa[a][u] = ldg_stream16(W + wrow_a + wbase);
                        sa[a][u] = ldg_u16(S + srow_a + grp);
                        ba[a][u] = ldg_u16(B + srow_a + grp);
                    }
                    if (kv[u] && vb) {
                        wb[a][u] = ldg_stream16(W + wrow_b + wbase);
                        sb[a][u] = ldg_u16(S + srow_b + grp);
                        bb[a][u] = ldg_u16(B + srow_b + grp);
                    }
                }
            }
            if (!waited) {
                pdl_wait();
                waited = true;
            }
            // token rows for the B fragments of this pass
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int m = m0 + 8 * nt + g;
                xrow[nt] = nullptr;
                if (m < Mp) {
                    const int64_t row = prm.x_rows ? (int64_t)prm.x_rows[off + m]
                                        : (prm.x_from_offset ? (int64_t)off + m
                                                             : (int64_t)xi * prm.M + m);
                    xrow[nt] = prm.x + row * prm.x_ld;
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int64_t kcode0 = ((int64_t)(kb0 + u) * 16 + 4 * c) * kCodesPerWord;
#pragma unroll
                for (int a = 0; a < NACC; ++a)
                    kblock_mma<BITS, NT>(acc[a], wa[a][u], wb[a][u], sa[a][u], ba[a][u], sb[a][u],
                                         bb[a][u], xrow, kcode0, kv[u]);
            }
        }
        if (!waited) {
            pdl_wait();
            waited = true;
        }

        // ---- reduce over the warps of this CTA
        float *mine = red + (size_t)warp * NACC * NT * 128;
#pragma unroll
        for (int a = 0; a < NACC; ++a)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) mine[((a * NT + nt) * 4 + j) * 32 + lane] = acc[a][nt][j];
        __syncthreads();
        if (warp == 0) {
            for (int w = 1; w < warps; ++w) {
                const float *o = red + (size_t)w * NACC * NT * 128;
#pragma unroll
                for (int a = 0; a < NACC; ++a)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            acc[a][nt][j] += o[((a * NT + nt) * 4 + j) * 32 + lane];
            }
        }
        // ---- reduce over the CTAs of the cluster (split K) via DSMEM
        if (gridDim.y > 1) {
            cg::cluster_group cl = cg::this_cluster();
            __syncthreads();
            if (warp == 0) {
#pragma unroll
                for (int a = 0; a < NACC; ++a)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            red[((a * NT + nt) * 4 + j) * 32 + lane] = acc[a][nt][j];
            }
            cl.sync();
            if (blockIdx.y == 0 && warp == 0) {
                for (unsigned r = 1; r < gridDim.y; ++r) {
                    const float *o = cl.map_shared_rank(red, r);
#pragma unroll
                    for (int a = 0; a < NACC; ++a)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                acc[a][nt][j] += o[((a * NT + nt) * 4 + j) * 32 + lane];
                }
            }
            cl.sync();
        }
        // ---- store
        if (blockIdx.y == 0 && warp == 0) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int m = m0 + 8 * nt + 2 * c + (j & 1);
                    const int64_t n = (j < 2) ? ra : rb;
                    if (m >= Mp || n >= prm.N) continue;
                    float v = acc[0][nt][j];
                    if (DUAL && prm.swiglu) v = silu_f32(v) * acc[NACC - 1][nt][j];
                    const int64_t row = prm.y_rows ? (int64_t)prm.y_rows[off + m] : (int64_t)off + m;
                    if (prm.out_f32)
                        static_cast<float *>(prm.y)[row * prm.y_ld + n] = v;
                    else
                        static_cast<uint16_t *>(prm.y)[row * prm.y_ld + n] = f32_to_bf16(v);
                }
            }
        }
        __syncthreads();
    }
}

template <int BITS, int NT, bool DUAL>
cudaError_t launch_variant(const GemvParams &prm, dim3 grid, int threads, int cluster,
                           cudaStream_t stream) {
    constexpr int NACC = DUAL ? 2 : 1;
    const size_t smem = (size_t)(threads / 32) * NACC * NT * 128 * sizeof(float);
    auto kern = qgemv_kernel<BITS, NT, DUAL>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (cluster > 1) {
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = 1;
        attrs[na].val.clusterDim.y = cluster;
        attrs[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, prm);
}

template <int BITS, bool DUAL>
cudaError_t dispatch_nt(const GemvParams &prm, int nt, dim3 grid, int threads, int cluster,
                        cudaStream_t stream) {
    switch (nt) {
        case 1: return launch_variant<BITS, 1, DUAL>(prm, grid, threads, cluster, stream);
        case 2: return launch_variant<BITS, 2, DUAL>(prm, grid, threads, cluster, stream);
        default: return launch_variant<BITS, 4, DUAL>(prm, grid, threads, cluster, stream);
    }
}

}  // namespace

cudaError_t launch_gemv(const GemvProblems &q, cudaStream_t stream) {
    GemvParams prm;
    prm.w = q.w;
    prm.s = q.s;
    prm.b = q.b;
    prm.w2 = q.w2 ? q.w2 : q.w;
    prm.s2 = q.s2 ? q.s2 : q.s;
    prm.b2 = q.b2 ? q.b2 : q.b;
    prm.N = q.N;
    prm.K = q.K;
    prm.Kw = q.K * q.bits / 32;
    prm.G = q.K / q.gs;
    prm.gs_shift = q.gs == 32 ? 5 : (q.gs == 64 ? 6 : 7);
    prm.x = q.x;
    prm.x_ld = q.x_ld;
    prm.P = q.P;
    prm.M = q.M;
    prm.E = q.E;
    prm.x_batch = q.x_batch;
    prm.expert = q.expert;
    prm.m_count = q.m_count;
    prm.m_offset = q.m_offset;
    prm.x_rows = q.x_rows;
    prm.lhs = q.lhs;
    prm.y_rows = q.y_rows;
    prm.expert_is_p = q.expert_is_p ? 1 : 0;
    prm.x_from_offset = q.x_from_offset ? 1 : 0;
    prm.y = q.y;
    prm.y_ld = q.y_ld;
    prm.out_f32 = q.out_f32;
    prm.swiglu = q.swiglu;
    prm.kb_total = (int)((prm.Kw + 15) / 16);
    prm.err = device_error_word();

    const int64_t row_tiles = (q.N + 15) / 16;
    const int sms = sm_count();
    // Warps per CTA and CTAs per cluster (split K): aim for >= 2 CTAs of work
    // per SM while keeping >= 2 k-blocks per warp.
    int warps = 8;
    while (warps > 2 && prm.kb_total < warps * 2) warps >>= 1;
    int cluster = 1;
    const int64_t ctas = row_tiles * (int64_t)q.P;
    while (cluster < 8 && ctas * cluster < 2 * sms &&
           prm.kb_total >= (int64_t)warps * cluster * 2 * 2)
        cluster <<= 1;
    const int max_m = std::max(1, q.max_m);
    const int nt = max_m <= 8 ? 1 : (max_m <= 16 ? 2 : 4);
    dim3 grid((unsigned)row_tiles, (unsigned)cluster, (unsigned)q.P);
    const bool dual = q.w2 != nullptr;
    if (q.bits == 4)
        return dual ? dispatch_nt<4, true>(prm, nt, grid, warps * 32, cluster, stream)
                    : dispatch_nt<4, false>(prm, nt, grid, warps * 32, cluster, stream);
    return dual ? dispatch_nt<8, true>(prm, nt, grid, warps * 32, cluster, stream)
                : dispatch_nt<8, false>(prm, nt, grid, warps * 32, cluster, stream);
}

}  // namespace nq
