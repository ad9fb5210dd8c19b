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

#include <cuda.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

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
    int x_div;      // > 0: problem p reads x batch p / x_div (pairs of top_k slots)
    void *y;
    int64_t y_ld;
    int out_f32, swiglu;
    int kb_total;   // k-blocks per row (16 words each), the last one possibly partial
    int kb_full;    // complete k-blocks per row
    int s_cta;      // K slices handled by the warps of one CTA (1, 2 or 4)
    int mx;         // tokens staged per pass (async path)
    unsigned int *err;
    PushDev push;   // tensor-parallel fan-out of the stores (n == 0: local only)
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

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma16816h(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Registers of one k-block of work for one warp: RT row tiles x rows {g, g+8}
// x NACC weight sets.  Scales and biases are kept as zero-extended 16-bit values.
template <int RT, int NACC>
struct KBlock {
    uint4 w[RT][2][NACC];
    uint32_t s[RT][2][NACC], b[RT][2][NACC];
};

// Row pointers of one warp (per row tile, row g / g+8, weight set).
template <int RT, int NACC>
struct RowPtrs {
    const uint4 *w[RT][2][NACC];      // packed words of the row, advanced to this lane's chunk
    const uint16_t *s[RT][2][NACC];   // group scales of the row
    const uint16_t *b[RT][2][NACC];
};

__device__ __forceinline__ uint32_t ldg_u16z(const uint16_t *p) {
    uint16_t r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return (uint32_t)r;
}

// Loads one k-block.  kb is the k-block index; grp the group index of this
// lane's codes in it.  No predicates: every row pointer is valid memory.
template <int RT, int NACC>
__device__ __forceinline__ void load_kblock(KBlock<RT, NACC> &blk, const RowPtrs<RT, NACC> &rp,
                                            int kb, int grp) {
#pragma unroll
    for (int t = 0; t < RT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
                blk.w[t][h][a] = ldg_stream16(rp.w[t][h][a] + (size_t)kb * 4);
                blk.s[t][h][a] = ldg_u16z(rp.s[t][h][a] + grp);
                blk.b[t][h][a] = ldg_u16z(rp.b[t][h][a] + grp);
            }
}

// The tail k-block (fewer than 16 words left in every row): chunks past the
// end of the row get zero codes and zero scale/bias, i.e. weight 0.
template <int RT, int NACC>
__device__ __forceinline__ void load_kblock_tail(KBlock<RT, NACC> &blk,
                                                 const RowPtrs<RT, NACC> &rp, int kb, int grp,
                                                 bool valid) {
#pragma unroll
    for (int t = 0; t < RT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
                blk.w[t][h][a] = make_uint4(0, 0, 0, 0);
                blk.s[t][h][a] = blk.b[t][h][a] = 0;
                if (valid) {
                    blk.w[t][h][a] = ldg_stream16(rp.w[t][h][a] + (size_t)kb * 4);
                    blk.s[t][h][a] = ldg_u16z(rp.s[t][h][a] + grp);
                    blk.b[t][h][a] = ldg_u16z(rp.b[t][h][a] + grp);
                }
            }
}

// Dequantizes and multiplies one k-block.  xoff: element offset of this lane's
// codes in the activation rows (k of its first code); xrow[nt]: the token row
// this lane supplies to n-tile nt.
//   4 bits: word i holds codes xoff+8i .. +7; the two mma steps use the pairs
//   (q0,q4),(q1,q5) and (q2,q6),(q3,q7), the activations the same pairs of x.
//   8 bits: word i holds codes xoff+4i .. +3; one mma step.
template <int BITS, int NT, int RT, int NACC>
__device__ __forceinline__ void compute_kblock(float (&acc)[RT][NACC][NT][4],
                                               const KBlock<RT, NACC> &blk,
                                               const uint16_t *const (&xrow)[NT], int xoff) {
    if constexpr (BITS == 4) {
        Dq4 dq[RT][2][NACC];
#pragma unroll
        for (int t = 0; t < RT; ++t)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    Dq4 &d = dq[t][h][a];
                    d.s2 = prmt(blk.s[t][h][a], 0u, 0x1010u);
                    d.b2 = prmt(blk.b[t][h][a], 0u, 0x1010u);
                    d.n2 = bf2_fma(d.s2, 0xC300C300u, 0x80008000u);  // exact -128*s
                }
        uint4 xr[4][NT];  // all activation loads of the k-block first
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) xr[i][nt] = ldg16(xrow[nt] + xoff + 8 * i);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t bx[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint4 xv = xr[i][nt];
                bx[nt][0] = prmt(xv.x, xv.z, 0x5410u);  // (x0, x4)
                bx[nt][1] = prmt(xv.x, xv.z, 0x7632u);  // (x1, x5)
                bx[nt][2] = prmt(xv.y, xv.w, 0x5410u);  // (x2, x6)
                bx[nt][3] = prmt(xv.y, xv.w, 0x7632u);  // (x3, x7)
            }
#pragma unroll
            for (int t = 0; t < RT; ++t)
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    const uint32_t wa = (&blk.w[t][0][a].x)[i];
                    const uint32_t wb = (&blk.w[t][1][a].x)[i];
                    const uint32_t wa4 = wa >> 4, wb4 = wb >> 4;
                    const uint32_t a0 = dq4_pair(lop3_and_or(wa, 0x000F000Fu, 0x43004300u), dq[t][0][a]);
                    const uint32_t a1 = dq4_pair(lop3_and_or(wb, 0x000F000Fu, 0x43004300u), dq[t][1][a]);
                    const uint32_t a2 = dq4_pair(lop3_and_or(wa4, 0x000F000Fu, 0x43004300u), dq[t][0][a]);
                    const uint32_t a3 = dq4_pair(lop3_and_or(wb4, 0x000F000Fu, 0x43004300u), dq[t][1][a]);
                    const uint32_t c0 = dq4_pair(lop3_and_or(wa >> 8, 0x000F000Fu, 0x43004300u), dq[t][0][a]);
                    const uint32_t c1 = dq4_pair(lop3_and_or(wb >> 8, 0x000F000Fu, 0x43004300u), dq[t][1][a]);
                    const uint32_t c2 = dq4_pair(lop3_and_or(wa4 >> 8, 0x000F000Fu, 0x43004300u), dq[t][0][a]);
                    const uint32_t c3 = dq4_pair(lop3_and_or(wb4 >> 8, 0x000F000Fu, 0x43004300u), dq[t][1][a]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        mma16816(acc[t][a][nt], a0, a1, a2, a3, bx[nt][0], bx[nt][1]);
                        mma16816(acc[t][a][nt], c0, c1, c2, c3, bx[nt][2], bx[nt][3]);
                    }
                }
        }
    } else {
        Dq8 dq[RT][2][NACC];
#pragma unroll
        for (int t = 0; t < RT; ++t)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int a = 0; a < NACC; ++a)
                    dq[t][h][a] = make_dq8((uint16_t)blk.s[t][h][a], (uint16_t)blk.b[t][h][a]);
        uint2 xr[4][NT];  // all activation loads of the k-block first
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) xr[i][nt] = ldg8(xrow[nt] + xoff + 4 * i);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint2 *bx = xr[i];
#pragma unroll
            for (int t = 0; t < RT; ++t)
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    const uint32_t wa = (&blk.w[t][0][a].x)[i];
                    const uint32_t wb = (&blk.w[t][1][a].x)[i];
                    const uint32_t a0 = dq8_pair(wa, 0, 1, dq[t][0][a]);
                    const uint32_t a1 = dq8_pair(wb, 0, 1, dq[t][1][a]);
                    const uint32_t a2 = dq8_pair(wa, 2, 3, dq[t][0][a]);
                    const uint32_t a3 = dq8_pair(wb, 2, 3, dq[t][1][a]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        mma16816(acc[t][a][nt], a0, a1, a2, a3, bx[nt].x, bx[nt].y);
                }
        }
    }
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

// Launch geometry chosen on the host (see launch_gemv):
//   blockDim 128 (4 warps).  A warp owns RT 16-row tiles ("a row group") of one
//   problem and one K slice.  s_cta warps of a CTA share a row group and split
//   its K (reduced in shared memory); gridDim.y CTAs of a cluster split it
//   further (reduced through distributed shared memory).
template <int BITS, int NT, int RT, bool DUAL>
__global__ void __launch_bounds__(128) qgemv_kernel(const GemvParams prm) {
    constexpr int NACC = DUAL ? 2 : 1;
    constexpr int kCodesPerKb = 16 * 32 / BITS;     // codes of one k-block (per row)
    constexpr int kCodesPerLane = 4 * 32 / BITS;    // codes of one lane's 16 bytes
    extern __shared__ float red[];                  // [4 warps][RT][NACC][NT][4][32]

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int p = blockIdx.z;
    const int s_cta = prm.s_cta;

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
    int xi = prm.lhs ? prm.lhs[p]
                     : (prm.x_div > 0 ? p / prm.x_div : (prm.x_batch == prm.P ? p : 0));
    if (xi < 0 || xi >= prm.x_batch) {
        bad = true;
        xi = 0;
    }
    if (bad && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
        atomicOr(prm.err, kErrBadIndex);
    if (Mp <= 0) return;  // uniform over the CTA and the cluster (same problem)

    const int slice_local = warp % s_cta;
    const int64_t rg = (int64_t)blockIdx.x * (4 / s_cta) + warp / s_cta;
    const int ksplit = gridDim.y * s_cta;
    const int slice = blockIdx.y * s_cta + slice_local;
    const int kb_lo = (int)(((int64_t)slice * prm.kb_total) / ksplit);
    const int kb_hi = (int)(((int64_t)(slice + 1) * prm.kb_total) / ksplit);
    const int kb_full_hi = min(kb_hi, prm.kb_full);

    // row pointers (rows past N are clamped to N-1: valid memory, never stored)
    RowPtrs<RT, NACC> rp;
    int64_t rows[RT][2];
#pragma unroll
    for (int t = 0; t < RT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            rows[t][h] = rg * (16 * RT) + 16 * t + 8 * h + g;
            const int64_t rc = min(rows[t][h], prm.N - 1) + (int64_t)e * prm.N;
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
                const uint32_t *W = a ? prm.w2 : prm.w;
                rp.w[t][h][a] = reinterpret_cast<const uint4 *>(W + rc * prm.Kw) + c;
                rp.s[t][h][a] = (a ? prm.s2 : prm.s) + rc * prm.G;
                rp.b[t][h][a] = (a ? prm.b2 : prm.b) + rc * prm.G;
            }
        }

    bool waited = indexed;
    for (int m0 = 0; m0 < Mp; m0 += 8 * NT) {
        float acc[RT][NACC][NT][4];
#pragma unroll
        for (int t = 0; t < RT; ++t)
#pragma unroll
            for (int a = 0; a < NACC; ++a)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[t][a][nt][j] = 0.0f;

        if (!bad) {
            const uint16_t *xrow[NT];
            KBlock<RT, NACC> A, B;
            int kb = kb_lo;
            if (kb < kb_full_hi) load_kblock(A, rp, kb, (kb * kCodesPerKb + c * kCodesPerLane) >> prm.gs_shift);
            if (!waited) {
                pdl_wait();
                waited = true;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int m = min(m0 + 8 * nt + g, Mp - 1);
                const int64_t row = prm.x_rows ? (int64_t)prm.x_rows[off + m]
                                    : (prm.x_from_offset ? (int64_t)off + m
                                                         : (int64_t)xi * prm.M + m);
                xrow[nt] = prm.x + row * prm.x_ld;
            }
            // main loop: full k-blocks, double-buffered in registers
            for (; kb < kb_full_hi; kb += 2) {
                if (kb + 1 < kb_full_hi)
                    load_kblock(B, rp, kb + 1, ((kb + 1) * kCodesPerKb + c * kCodesPerLane) >> prm.gs_shift);
                compute_kblock<BITS, NT, RT, NACC>(acc, A, xrow, kb * kCodesPerKb + c * kCodesPerLane);
                if (kb + 1 >= kb_full_hi) break;
                if (kb + 2 < kb_full_hi)
                    load_kblock(A, rp, kb + 2, ((kb + 2) * kCodesPerKb + c * kCodesPerLane) >> prm.gs_shift);
                compute_kblock<BITS, NT, RT, NACC>(acc, B, xrow, (kb + 1) * kCodesPerKb + c * kCodesPerLane);
            }
            // the partial last k-block, if this slice holds it
            if (kb_hi > prm.kb_full) {
                const int kt = prm.kb_full;
                const bool valid = (int64_t)kt * 16 + 4 * c + 4 <= prm.Kw;
                const int code0 = kt * kCodesPerKb + c * kCodesPerLane;
                load_kblock_tail(A, rp, kt, code0 >> prm.gs_shift, valid);
                compute_kblock<BITS, NT, RT, NACC>(acc, A, xrow, valid ? code0 : 0);
            }
        } else if (!waited) {
            pdl_wait();
            waited = true;
        }

        // ---- reduce the K slices of the CTA (shared memory)
        constexpr int kVals = RT * NACC * NT * 4;
        if (s_cta > 1) {
            float *mine = red + (size_t)warp * kVals * 32;
#pragma unroll
            for (int t = 0; t < RT; ++t)
#pragma unroll
                for (int a = 0; a < NACC; ++a)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            mine[(((t * NACC + a) * NT + nt) * 4 + j) * 32 + lane] = acc[t][a][nt][j];
            __syncthreads();
            if (slice_local == 0) {
                for (int w = 1; w < s_cta; ++w) {
                    const float *o = red + (size_t)(warp + w) * kVals * 32;
#pragma unroll
                    for (int t = 0; t < RT; ++t)
#pragma unroll
                        for (int a = 0; a < NACC; ++a)
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                                for (int j = 0; j < 4; ++j)
                                    acc[t][a][nt][j] += o[(((t * NACC + a) * NT + nt) * 4 + j) * 32 + lane];
                }
            }
        }
        // ---- reduce across the CTAs of the cluster (distributed shared memory)
        if (gridDim.y > 1) {
            cg::cluster_group cl = cg::this_cluster();
            if (s_cta > 1) __syncthreads();
            float *mine = red + (size_t)warp * kVals * 32;
            if (slice_local == 0) {
#pragma unroll
                for (int t = 0; t < RT; ++t)
#pragma unroll
                    for (int a = 0; a < NACC; ++a)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                mine[(((t * NACC + a) * NT + nt) * 4 + j) * 32 + lane] = acc[t][a][nt][j];
            }
            cl.sync();
            if (blockIdx.y == 0 && slice_local == 0) {
                for (unsigned r = 1; r < gridDim.y; ++r) {
                    const float *o = cl.map_shared_rank(mine, r);
#pragma unroll
                    for (int t = 0; t < RT; ++t)
#pragma unroll
                        for (int a = 0; a < NACC; ++a)
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                                for (int j = 0; j < 4; ++j)
                                    acc[t][a][nt][j] += o[(((t * NACC + a) * NT + nt) * 4 + j) * 32 + lane];
                }
            }
            cl.sync();
        }
        // ---- store
        if (blockIdx.y == 0 && slice_local == 0) {
#pragma unroll
            for (int t = 0; t < RT; ++t)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int m = m0 + 8 * nt + 2 * c + (j & 1);
                        const int64_t n = rows[t][j >> 1];
                        if (m >= Mp || n >= prm.N) continue;
                        float v = acc[t][0][nt][j];
                        if (DUAL && prm.swiglu) v = silu_f32(v) * acc[t][NACC - 1][nt][j];
                        const int64_t row = prm.y_rows ? (int64_t)prm.y_rows[off + m] : (int64_t)off + m;
                        if (prm.out_f32)
                            static_cast<float *>(prm.y)[row * prm.y_ld + n] = v;
                        else
                            static_cast<uint16_t *>(prm.y)[row * prm.y_ld + n] = f32_to_bf16(v);
                    }
        }
        if (s_cta > 1 && m0 + 8 * NT < Mp) __syncthreads();
    }
}

template <int BITS, int NT, int RT, bool DUAL>
cudaError_t launch_variant(const GemvParams &prm, dim3 grid, int cluster, cudaStream_t stream) {
    constexpr int NACC = DUAL ? 2 : 1;
    const size_t smem = (prm.s_cta > 1 || cluster > 1)
                            ? (size_t)4 * RT * NACC * NT * 4 * 32 * sizeof(float)
                            : 0;
    auto kern = qgemv_kernel<BITS, NT, RT, DUAL>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(128, 1, 1);
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
cudaError_t dispatch(const GemvParams &prm, int nt, int rt, dim3 grid, int cluster,
                     cudaStream_t stream) {
    if (nt == 1)
        return rt == 2 ? launch_variant<BITS, 1, 2, DUAL>(prm, grid, cluster, stream)
                       : launch_variant<BITS, 1, 1, DUAL>(prm, grid, cluster, stream);
    if (nt == 2) return launch_variant<BITS, 2, 1, DUAL>(prm, grid, cluster, stream);
    return launch_variant<BITS, 4, 1, DUAL>(prm, grid, cluster, stream);
}

// ----------------------------------------------------------------------------
// Asynchronously fed variant (the default path).  A CTA owns 64 weight rows
// (4 consumer warps x 16 rows) of one problem and one K slice.  Warp 4 fills a
// 4-stage shared-memory ring; one stage covers 32 packed words per row (256
// codes at 4 bits, 128 at 8 bits) and holds everything the consumers need for
// it, so they never wait on a global load:
//   * the packed words: one cp.async.bulk.tensor box [32 words x 64 rows] per
//     weight set, 128-byte swizzle (consumer reads are <= 2-way conflicted);
//   * the activation slice [mx tokens x stage codes] (cp.async, 16-byte
//     chunks, chunk index XOR token so the 8 token rows of a fragment hit
//     different banks; tokens past the problem's count are zero-filled);
//   * the scale and bias spans of the stage's groups for all 64 rows (cp.async).
// Completion: the bulk copies count bytes on the stage's mbarrier, and every
// producer lane's cp.asyncs arrive on it (cp.async.mbarrier.arrive.noinc).
// Consumers dequantize exactly (as the register path does), multiply with
// mma.sync into two independent accumulator chains, and release the stage.
// Requires K % 256 == 0 and (8-bit) group size <= 64; else the register path.
// ----------------------------------------------------------------------------
constexpr int kTStageWords = 32;   // packed words per row per stage
constexpr int kTConsumers = 4;     // consumer warps; each owns 16 * RT rows

// Byte layout of one stage (offsets from the stage base; base 1024-aligned).
struct TStageLayout {
    int set_bytes, x_off, x_row_bytes, s_off, s_row_bytes, bytes;
};

__host__ __device__ inline TStageLayout tstage_layout(int bits, int nacc, int rows, int mx, int gs) {
    TStageLayout L;
    const int codes = kTStageWords * 32 / bits;
    L.set_bytes = rows * kTStageWords * 4;
    L.x_off = nacc * L.set_bytes;
    L.x_row_bytes = codes * 2;
    L.s_off = L.x_off + mx * L.x_row_bytes;
    L.s_row_bytes = (codes / gs) * 2;       // one row's group span (4, 8 or 16 bytes) ...
    const int s_bytes = nacc * 2 * rows * 16;  // ... in a 16-byte slot: [set][scale|bias][row]
    L.bytes = (L.s_off + s_bytes + 1023) & ~1023;
    return L;
}

// Ring depth: 3 stages for 32-row warps and for the gate/up pair (their
// stages are twice as large), 4 otherwise -- sized so that the 128-row and
// paired kernels fit three CTAs per SM.
__host__ __device__ constexpr int tstages(int rt, bool dual) { return rt == 2 || dual ? 3 : 4; }

__device__ __forceinline__ bool tma_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                         unsigned int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            *abort = 1;
            atomicOr(err, kErrWaitTimeout);
            return false;
        }
    }
}

// cp.async of `bytes` (4, 8 or 16) from global to shared; src_bytes 0 zero-fills.
__device__ __forceinline__ void cp_async(void *dst, const void *src, int bytes, int src_bytes) {
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)),
                     "l"(src), "r"(src_bytes)
                     : "memory");
    else if (bytes == 8)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)),
                     "l"(src), "r"(src_bytes)
                     : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)),
                     "l"(src), "r"(src_bytes)
                     : "memory");
}

// The mbarrier receives one arrival once all prior cp.asyncs of this thread land.
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// One k-block from shared memory.  w[t][h][a]: this lane's 16 bytes of row h
// of tile t of weight set a; sv/bv: its rows' scale and bias bits; xo[nt][i]:
// byte offsets (in the stage's activation slice xs) of the 16-byte (4-bit) /
// 8-byte (8-bit) activation chunks this lane feeds to n-tile nt.
template <int BITS, int NT, int RT, int NACC>
__device__ __forceinline__ void compute_kb_smem(float (&acc)[2][RT][NACC][NT][4],
                                                const uint4 (&w)[RT][2][NACC],
                                                const uint32_t (&sv)[RT][2][NACC],
                                                const uint32_t (&bv)[RT][2][NACC],
                                                const uint8_t *xs, const int (&xo)[NT][4]) {
    if constexpr (BITS == 4) {
        Dq4 dq[RT][2][NACC];
#pragma unroll
        for (int t = 0; t < RT; ++t)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    dq[t][h][a].s2 = prmt(sv[t][h][a], 0u, 0x1010u);
                    dq[t][h][a].b2 = prmt(bv[t][h][a], 0u, 0x1010u);
                    dq[t][h][a].n2 = bf2_fma(dq[t][h][a].s2, 0xC300C300u, 0x80008000u);
                }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t bx[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint4 xv = *reinterpret_cast<const uint4 *>(xs + xo[nt][i]);
                bx[nt][0] = prmt(xv.x, xv.z, 0x5410u);  // (x0, x4)
                bx[nt][1] = prmt(xv.x, xv.z, 0x7632u);  // (x1, x5)
                bx[nt][2] = prmt(xv.y, xv.w, 0x5410u);  // (x2, x6)
                bx[nt][3] = prmt(xv.y, xv.w, 0x7632u);  // (x3, x7)
            }
#pragma unroll
            for (int t = 0; t < RT; ++t)
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    const uint32_t wa = (&w[t][0][a].x)[i];
                    const uint32_t wb = (&w[t][1][a].x)[i];
                    const uint32_t wa4 = wa >> 4, wb4 = wb >> 4;
                    const uint32_t a0 = dq4_pair(lop3_and_or(wa, 0x000F000Fu, 0x43004300u), dq[t][0][a]);
                    const uint32_t a1 = dq4_pair(lop3_and_or(wb, 0x000F000Fu, 0x43004300u), dq[t][1][a]);
                    const uint32_t a2 = dq4_pair(lop3_and_or(wa4, 0x000F000Fu, 0x43004300u), dq[t][0][a]);
                    const uint32_t a3 = dq4_pair(lop3_and_or(wb4, 0x000F000Fu, 0x43004300u), dq[t][1][a]);
                    const uint32_t c0 = dq4_pair(lop3_and_or(wa >> 8, 0x000F000Fu, 0x43004300u), dq[t][0][a]);
                    const uint32_t c1 = dq4_pair(lop3_and_or(wb >> 8, 0x000F000Fu, 0x43004300u), dq[t][1][a]);
                    const uint32_t c2 = dq4_pair(lop3_and_or(wa4 >> 8, 0x000F000Fu, 0x43004300u), dq[t][0][a]);
                    const uint32_t c3 = dq4_pair(lop3_and_or(wb4 >> 8, 0x000F000Fu, 0x43004300u), dq[t][1][a]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        mma16816(acc[0][t][a][nt], a0, a1, a2, a3, bx[nt][0], bx[nt][1]);
                        mma16816(acc[1][t][a][nt], c0, c1, c2, c3, bx[nt][2], bx[nt][3]);
                    }
                }
        }
    } else {
        Dq8 dq[RT][2][NACC];
#pragma unroll
        for (int t = 0; t < RT; ++t)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int a = 0; a < NACC; ++a)
                    dq[t][h][a] = make_dq8((uint16_t)sv[t][h][a], (uint16_t)bv[t][h][a]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint2 bx[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                bx[nt] = *reinterpret_cast<const uint2 *>(xs + xo[nt][i]);
#pragma unroll
            for (int t = 0; t < RT; ++t)
#pragma unroll
                for (int a = 0; a < NACC; ++a) {
                    const uint32_t wa = (&w[t][0][a].x)[i];
                    const uint32_t wb = (&w[t][1][a].x)[i];
                    const uint32_t a0 = dq8_pair(wa, 0, 1, dq[t][0][a]);
                    const uint32_t a1 = dq8_pair(wb, 0, 1, dq[t][1][a]);
                    const uint32_t a2 = dq8_pair(wa, 2, 3, dq[t][0][a]);
                    const uint32_t a3 = dq8_pair(wb, 2, 3, dq[t][1][a]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        mma16816(acc[i & 1][t][a][nt], a0, a1, a2, a3, bx[nt].x, bx[nt].y);
                }
        }
    }
}

template <int BITS, int NT, int RT, bool DUAL>
__global__ void __launch_bounds__(160) qgemv_tma_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                        const __grid_constant__ CUtensorMap tm_w2,
                                                        const GemvParams prm) {
    constexpr int NACC = DUAL ? 2 : 1;
    constexpr int kRows = kTConsumers * 16 * RT;  // weight rows per CTA
    constexpr int kStages = tstages(RT, DUAL);
    constexpr int kCodesPerStage = kTStageWords * 32 / BITS;
    constexpr int kCodesPerKb = 16 * 32 / BITS;
    constexpr int kCodesPerLane = 4 * 32 / BITS;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    const int mx = prm.mx;
    const TStageLayout L = tstage_layout(BITS, NACC, kRows, mx, 1 << prm.gs_shift);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * L.bytes);
    uint64_t *empty = full + kStages;
    volatile int *abort = reinterpret_cast<volatile int *>(empty + kStages);
    float *red = reinterpret_cast<float *>(smem + kStages * L.bytes + 128);

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int p = blockIdx.z;

    pdl_launch_dependents();
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
    int xi = prm.lhs ? prm.lhs[p]
                     : (prm.x_div > 0 ? p / prm.x_div : (prm.x_batch == prm.P ? p : 0));
    if (xi < 0 || xi >= prm.x_batch) {
        bad = true;
        xi = 0;
    }
    if (bad && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
        atomicOr(prm.err, kErrBadIndex);
    if (Mp <= 0) return;  // uniform over the CTA and the cluster (same problem)

    const int n_stg_total = (int)(prm.K / kCodesPerStage);
    const int ksplit = gridDim.y;
    const int st_lo = (int)(((int64_t)blockIdx.y * n_stg_total) / ksplit);
    const int st_hi = (int)(((int64_t)(blockIdx.y + 1) * n_stg_total) / ksplit);
    const int nst = bad ? 0 : st_hi - st_lo;
    const int passes = (Mp + mx - 1) / mx;
    const int64_t n_base = (int64_t)blockIdx.x * kRows;
    if (gridDim.y > 1 && passes > 1) {
        // never launched this way (the host splits K only when every problem
        // fits one pass); refuse rather than risk the cluster barriers
        if (threadIdx.x == 0) atomicOr(prm.err, kErrBadIndex);
        return;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1 + 32);  // producer expect_tx + 32 cp.async lanes
            mbar_init(&empty[s], kTConsumers);
        }
        *abort = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kTConsumers) {
        // ------------------------------------------------------ producer warp
        // Weights and scales never depend on the previous kernel on the stream,
        // activations may: the first ring of weight boxes and scale spans is
        // issued before griddepcontrol.wait, so with programmatic dependent
        // launch this projection's weight stream overlaps the previous kernel.
        const int total = nst * passes;
        const int32_t row0 = (int32_t)((int64_t)e * prm.N + n_base);
        const int chunks = L.x_row_bytes / 16;  // 16-byte chunks per token row
        auto issue_weights = [&](int t) {
            const int s = t % kStages;
            uint8_t *st = smem + s * L.bytes;
            const int pass = t / nst;
            const int stage = st_lo + (t - pass * nst);
            if (lane == 0) {
                mbar_expect_tx(&full[s], NACC * L.set_bytes);
                tma_load_2d(st, &tm_w, &full[s], stage * kTStageWords, row0);
                if (DUAL) tma_load_2d(st + L.set_bytes, &tm_w2, &full[s], stage * kTStageWords, row0);
            }
            const int grp0 = (stage * kCodesPerStage) >> prm.gs_shift;
            for (int q = lane; q < NACC * 2 * kRows; q += 32) {
                const int a = q / (2 * kRows), sb = (q / kRows) & 1, r = q % kRows;
                const int64_t rc = min(n_base + r, prm.N - 1) + (int64_t)e * prm.N;
                const uint16_t *base = sb ? (a ? prm.b2 : prm.b) : (a ? prm.s2 : prm.s);
                cp_async(st + L.s_off + q * 16, base + rc * prm.G + grp0, L.s_row_bytes,
                         L.s_row_bytes);
            }
        };
        // The activation row of token tk of the current pass, held by lane tk
        // (mx <= 32): looked up once per pass, not once per stage.
        int cached_pass = -1;
        int64_t lane_row = 0;
        auto issue_acts = [&](int t) {
            const int s = t % kStages;
            uint8_t *st = smem + s * L.bytes;
            const int pass = t / nst;
            const int stage = st_lo + (t - pass * nst);
            const int m0 = pass * mx;
            const int code0 = stage * kCodesPerStage;
            if (pass != cached_pass) {  // uniform over the warp
                const int m = m0 + lane;
                lane_row = 0;
                if (lane < mx && m < Mp)
                    lane_row = prm.x_rows ? (int64_t)prm.x_rows[off + m]
                                          : (prm.x_from_offset ? (int64_t)off + m
                                                               : (int64_t)xi * prm.M + m);
                cached_pass = pass;
            }
            for (int tk = 0; tk < mx; ++tk) {
                const int m = m0 + tk;
                const uint16_t *src = prm.x;
                int nbytes = 0;
                const int64_t row = __shfl_sync(0xffffffffu, lane_row, tk);
                if (m < Mp) {
                    src = prm.x + row * prm.x_ld + code0;
                    nbytes = 16;
                }
                uint8_t *xdst = st + L.x_off + tk * L.x_row_bytes;
                for (int ch = lane; ch < chunks; ch += 32)
                    cp_async(xdst + ((ch ^ (tk & 7)) << 4), src + (nbytes ? ch * 8 : 0), 16, nbytes);
            }
            cp_async_arrive(&full[s]);  // this lane's copies of the stage, weights included
        };
        int t = 0;
        if (nst > 0) {
            if (lane == 0) {
                prefetch_tmap(&tm_w);
                if (DUAL) prefetch_tmap(&tm_w2);
            }
            const int pre = min(total, kStages);  // ring slots free at start: no wait
            for (int u = 0; u < pre; ++u) issue_weights(u);
            if (!indexed) pdl_wait();
            for (int u = 0; u < pre; ++u) issue_acts(u);
            for (t = pre; t < total; ++t) {
                const int s = t % kStages;
                const uint32_t ph = (uint32_t)(t / kStages) & 1u;
                // the whole warp stops together (issue_acts shuffles across it)
                if (!__all_sync(0xffffffffu, tma_wait(&empty[s], ph ^ 1u, abort, prm.err))) break;
                issue_weights(t);
                issue_acts(t);
            }
            // every issued copy must land before the CTA may exit
            for (int u = (t > kStages ? t - kStages : 0); u < t; ++u)
                tma_wait(&full[u % kStages], (uint32_t)(u / kStages) & 1u, abort, prm.err);
        }
        __syncwarp();
        // Cluster K split (only ever launched with a single token pass): the
        // consumers meet twice per pass; the producer has issued every stage by
        // then, so it can join without blocking them.
        if (gridDim.y > 1) {
            cg::cluster_group cl = cg::this_cluster();
            for (int pass = 0; pass < passes; ++pass) {
                cl.sync();
                cl.sync();
            }
        }
    } else {
        // ------------------------------------------------------ consumer warps
        // Every shared-memory read is (per-lane base) + (compile-time constant):
        //   packed words of row warp*16*RT + 16r + 8h + g: the 128-byte swizzle
        //   XORs the chunk with (row & 7) == g, so only the k-block term is
        //   lane-dependent; scales/biases sit in 16-byte row slots.
        const int row_l = warp * 16 * RT + g;
        const int wbase0 = row_l * 128 + (((0 + c) ^ g) << 4);
        const int wbase1 = row_l * 128 + (((4 + c) ^ g) << 4);
        const int gl0 = (c * kCodesPerLane) >> prm.gs_shift;
        const int gl1 = (kCodesPerKb + c * kCodesPerLane) >> prm.gs_shift;
        const int sbase0 = L.s_off + row_l * 16 + gl0 * 2;
        const int sbase1 = L.s_off + row_l * 16 + gl1 * 2;
        int t = 0;
        for (int pass = 0; pass < passes; ++pass) {
            const int m0 = pass * mx;
            int xo[NT][4];  // activation chunk offsets of k-block 0 (k-block 1: + kb bytes)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int tk = min(8 * nt + g, mx - 1);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int el = c * kCodesPerLane + i * (32 / BITS);
                    xo[nt][i] = L.x_off + tk * L.x_row_bytes + (((el >> 3) ^ (tk & 7)) << 4) +
                                ((el & 7) << 1);
                }
            }
            float acc[2][RT][NACC][NT][4];
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int r = 0; r < RT; ++r)
#pragma unroll
                    for (int a = 0; a < NACC; ++a)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int j = 0; j < 4; ++j) acc[u][r][a][nt][j] = 0.0f;

            for (int i = 0; i < nst; ++i, ++t) {
                const int s = t % kStages;
                const uint32_t ph = (uint32_t)(t / kStages) & 1u;
                if (!tma_wait(&full[s], ph, abort, prm.err)) break;
                const uint8_t *st = smem + s * L.bytes;
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    const uint8_t *wb = st + (kk ? wbase1 : wbase0);
                    const uint8_t *sb = st + (kk ? sbase1 : sbase0);
                    uint4 w[RT][2][NACC];
                    uint32_t sv[RT][2][NACC], bv[RT][2][NACC];
#pragma unroll
                    for (int r = 0; r < RT; ++r)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
#pragma unroll
                            for (int a = 0; a < NACC; ++a) {
                                constexpr int kSet = kRows * kTStageWords * 4;
                                const int ro = (16 * r + 8 * h);
                                w[r][h][a] = *reinterpret_cast<const uint4 *>(wb + a * kSet + ro * 128);
                                sv[r][h][a] = *reinterpret_cast<const uint16_t *>(
                                    sb + (a * 2 + 0) * kRows * 16 + ro * 16);
                                bv[r][h][a] = *reinterpret_cast<const uint16_t *>(
                                    sb + (a * 2 + 1) * kRows * 16 + ro * 16);
                            }
                    compute_kb_smem<BITS, NT, RT, NACC>(acc, w, sv, bv, st + kk * kCodesPerKb * 2,
                                                       xo);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            // fold the two accumulator chains
#pragma unroll
            for (int r = 0; r < RT; ++r)
#pragma unroll
                for (int a = 0; a < NACC; ++a)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[0][r][a][nt][j] += acc[1][r][a][nt][j];
            // ---- reduce the K slices of the cluster (distributed shared memory)
            constexpr int kVals = RT * NACC * NT * 4;
            float *mine = red + (size_t)warp * kVals * 32;
            if (gridDim.y > 1) {
                cg::cluster_group cl = cg::this_cluster();
#pragma unroll
                for (int r = 0; r < RT; ++r)
#pragma unroll
                    for (int a = 0; a < NACC; ++a)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                mine[(((r * NACC + a) * NT + nt) * 4 + j) * 32 + lane] =
                                    acc[0][r][a][nt][j];
                cl.sync();  // the producer warp joins both cluster barriers of a pass
                if (blockIdx.y == 0) {
                    for (unsigned q = 1; q < gridDim.y; ++q) {
                        const float *o = cl.map_shared_rank(mine, q);
#pragma unroll
                        for (int r = 0; r < RT; ++r)
#pragma unroll
                            for (int a = 0; a < NACC; ++a)
#pragma unroll
                                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                                    for (int j = 0; j < 4; ++j)
                                        acc[0][r][a][nt][j] +=
                                            o[(((r * NACC + a) * NT + nt) * 4 + j) * 32 + lane];
                    }
                }
                cl.sync();
            }
            if (!indexed) pdl_wait();  // (no-op once the producer's copies landed)
            bool store_ok = true;
            if (prm.push.n && blockIdx.y == 0) store_ok = push_wait_ready(prm.push, prm.err);
            if (blockIdx.y == 0 && store_ok) {
#pragma unroll
                for (int r = 0; r < RT; ++r)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int m = m0 + 8 * nt + 2 * c + (j & 1);
                            const int64_t n = n_base + warp * 16 * RT + 16 * r + g + 8 * (j >> 1);
                            if (m >= Mp || m >= m0 + mx || n >= prm.N) continue;
                            float v = acc[0][r][0][nt][j];
                            if (DUAL && prm.swiglu) v = silu_f32(v) * acc[0][r][NACC - 1][nt][j];
                            const int64_t row =
                                prm.y_rows ? (int64_t)prm.y_rows[off + m] : (int64_t)off + m;
                            if (prm.out_f32)
                                push_store(prm.push, static_cast<float *>(prm.y) + row * prm.y_ld + n,
                                           v);
                            else
                                push_store(prm.push,
                                           static_cast<uint16_t *>(prm.y) + row * prm.y_ld + n,
                                           f32_to_bf16(v));
                        }
            }
        }
    }
}

template <int BITS, int NT, int RT, bool DUAL>
cudaError_t launch_tma_variant(const CUtensorMap &m1, const CUtensorMap &m2,
                               const GemvParams &prm, dim3 grid, int cluster,
                               cudaStream_t stream) {
    constexpr int NACC = DUAL ? 2 : 1;
    constexpr int kRows = kTConsumers * 16 * RT;
    const TStageLayout L = tstage_layout(BITS, NACC, kRows, prm.mx, 1 << prm.gs_shift);
    // the K-slice partial sums are only exchanged inside a cluster
    const int red_bytes = cluster > 1 ? kTConsumers * RT * NACC * NT * 4 * 32 * 4 : 0;
    const int smem = tstages(RT, DUAL) * L.bytes + 1024 + 128 + red_bytes;
    auto kern = qgemv_tma_kernel<BITS, NT, RT, DUAL>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(32 * (kTConsumers + 1), 1, 1);
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
    return cudaLaunchKernelEx(&cfg, kern, m1, m2, prm);
}

template <int BITS, bool DUAL>
cudaError_t dispatch_tma(const CUtensorMap &m1, const CUtensorMap &m2, const GemvParams &prm,
                         int nt, int rt, dim3 grid, int cluster, cudaStream_t stream) {
    if (nt == 1)
        return rt == 2 ? launch_tma_variant<BITS, 1, 2, DUAL>(m1, m2, prm, grid, cluster, stream)
                       : launch_tma_variant<BITS, 1, 1, DUAL>(m1, m2, prm, grid, cluster, stream);
    if (nt == 2) return launch_tma_variant<BITS, 2, 1, DUAL>(m1, m2, prm, grid, cluster, stream);
    return launch_tma_variant<BITS, 4, 1, DUAL>(m1, m2, prm, grid, cluster, stream);
}

// ----------------------------------------------------------------------------
// Row-group kernel for plain decode problems (one problem, M <= 8 tokens,
// 4-bit codes, K a multiple of 128).  A CTA owns one group of 16 weight rows
// and all of K; its W warps split K exactly: warp w owns k-blocks
// [w*KBW, (w+1)*KBW) (a k-block is 16 packed words, 128 codes, per row).
//   * Every lane loads its whole share of the weights (2 rows x KBW x 16 bytes)
//     and its scale/bias values straight into registers before
//     griddepcontrol.wait, so with programmatic dependent launch the weight
//     stream of one projection runs under the tail of the previous kernel.
//     Nothing else is in flight on the critical path: no ring, no cluster.
//   * PAIR: a CTA takes two groups; the second group's rows, scales and
//     biases travel by untiled bulk copies into shared memory (one mbarrier,
//     bounded wait), also issued before griddepcontrol.wait.  Used when that
//     is what lets every CTA of the launch be resident at once (rows_plan).
//   * After the wait each warp copies its slice of x into its own shared
//     memory (all of a lane's global reads issued at once: its x chunks, the
//     prologue's second operand, the residual it will add), pairs permuted
//     to the order of the mma.sync B fragments
//     ((x0,x4),(x1,x5),(x2,x6),(x3,x7)) and chunks laid out so that the four
//     lanes of a row read consecutive 16-byte chunks.
//   * The unrolled main loop dequantizes exactly (as the kernels above) into
//     mma.sync A fragments; the K-slices are summed in shared memory.
//   * Optional prologue in the staging of x (RMSNorm of the row, or SwiGLU of
//     a [gate | up] row) and residual epilogue (launch_rows_fused): the decode
//     step's norms, activation and residual adds run inside its GEMVs.
// Measured (B200, CUDA graph of back-to-back calls on weight sets larger than
// L2): 4096x4096 at M=1 6.0 us (the TMA-fed kernel: 7.9 us); 256x4096 3.3 us,
// the part that does not shrink with the weights.
// ----------------------------------------------------------------------------
constexpr int kRowsPlain = 0, kRowsNorm = 1, kRowsSwiglu = 2;

struct RowsParams {
    const uint32_t *w;
    const uint16_t *s, *b, *x;
    uint16_t *y;
    int64_t N, K, Kw, G, x_ld, y_ld;
    int gs_shift, M;
    // prologue applied to each x row as it is staged (kRowsPlain for none)
    int pro;
    const uint16_t *nw;  // kRowsNorm: the RMSNorm weight [K]
    float eps;
    // epilogue: y = bf16(res + bf16(acc)) when res != nullptr (rows res_ld apart)
    const uint16_t *res;
    int64_t res_ld;
    unsigned int *err;  // device error word (bounded-wait timeouts)
    // epi_swiglu (M == 1): every group of 16 rows is 8 gate rows followed by
    // the 8 matching up rows; the output is y[8 * group + i] =
    // swiglu(bf16(gate_i), bf16(up_i)) (N / 2 values)
    int epi_swiglu;
};

// x = bf16(bf16(bf16(sigmoid(g)) * g) * u) for one bf16 pair each of g, u:
// the SwiGLU op chain of mlx_ops' callers (sigmoid(gate) * gate * up, each
// op rounded to bf16)
__device__ __forceinline__ uint32_t swiglu_pair(uint32_t g2, uint32_t u2) {
    uint32_t out = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float g = bf16_to_f32((uint16_t)(g2 >> (16 * h)));
        const float u = bf16_to_f32((uint16_t)(u2 >> (16 * h)));
        const float sg = bf16_to_f32(f32_to_bf16(1.0f / (1.0f + expf(-g))));
        const float a = bf16_to_f32(f32_to_bf16(sg * g));
        out |= (uint32_t)f32_to_bf16(a * u) << (16 * h);
    }
    return out;
}

// y = bf16(w * bf16(x * inv)) for one bf16 pair each of x, w (MLX's rms_norm
// output rounding)
__device__ __forceinline__ uint32_t norm_pair(uint32_t x2, uint32_t w2, float inv) {
    uint32_t out = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float x = bf16_to_f32((uint16_t)(x2 >> (16 * h)));
        const float w = bf16_to_f32((uint16_t)(w2 >> (16 * h)));
        out |= (uint32_t)f32_to_bf16(w * bf16_to_f32(f32_to_bf16(x * inv))) << (16 * h);
    }
    return out;
}

__device__ __forceinline__ uint4 pair_permute(uint4 v) {
    uint4 o;
    o.x = prmt(v.x, v.z, 0x5410u);
    o.y = prmt(v.x, v.z, 0x7632u);
    o.z = prmt(v.y, v.w, 0x5410u);
    o.w = prmt(v.y, v.w, 0x7632u);
    return o;
}

template <int KBW, bool F16, bool PAIR>
__global__ void __launch_bounds__(512) qgemv_rows_kernel(const RowsParams p) {
    constexpr int XCH = KBW * 16;  // 16-byte x chunks per token in a warp's slice
    extern __shared__ __align__(128) uint4 rows_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int W = blockDim.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int M = p.M;
    uint4 *xs = rows_smem + (size_t)warp * M * XCH;                        // [M][XCH]
    float *red = reinterpret_cast<float *>(rows_smem + (size_t)W * M * XCH);  // [W][4][32]
    pdl_launch_dependents();
    const int kb0 = warp * KBW;
    const int64_t r0 = (int64_t)blockIdx.x * (PAIR ? 32 : 16);
    // PAIR: the CTA's second group of 16 rows (r0 + 16 ...) travels by bulk
    // copies into shared memory, issued here, before the dependency wait, so
    // that its weights stream beside the first group's register loads.
    // Layout after red: 16 rows of packed codes (row stride rs bytes, padded
    // so that the two rows a quarter-warp reads fall in different banks),
    // then 16 rows of scales and 16 of biases (G * 2 bytes each), then the
    // mbarrier.
    const int64_t rs = (p.K / 2) + (((p.K / 2) & 127) == 0 ? 64 : 0);
    uint8_t *bsm = reinterpret_cast<uint8_t *>(red + W * 4 * 32);
    uint8_t *bss = bsm + 16 * rs;
    uint8_t *bsb = bss + 16 * p.G * 2;
    uint64_t *bbar = reinterpret_cast<uint64_t *>(bsb + 16 * p.G * 2);
    if constexpr (PAIR) {
        if (threadIdx.x == 0) {
            mbar_init(bbar, 1);
            fence_barrier_init();
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            mbar_expect_tx(bbar, (uint32_t)(16 * (p.K / 2 + 4 * p.G)));
            for (int h = 0; h < 16; ++h) {
                // rows past N copy row N-1 (valid memory) and are never stored
                const int64_t row = min(r0 + 16 + h, p.N - 1);
                bulk_g2s(bsm + h * rs, p.w + row * p.Kw, (uint32_t)(p.K / 2), bbar);
                bulk_g2s(bss + h * p.G * 2, p.s + row * p.G, (uint32_t)(p.G * 2), bbar);
                bulk_g2s(bsb + h * p.G * 2, p.b + row * p.G, (uint32_t)(p.G * 2), bbar);
            }
        }
    }
    uint4 wv[KBW][2];
    uint32_t sb[KBW][2];  // scale | bias << 16
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        // rows past N read row N-1 (valid memory) and are never stored
        const int64_t row = min(r0 + 8 * h + g, p.N - 1);
        const uint32_t *wr = p.w + row * p.Kw + kb0 * 16 + 4 * c;
#pragma unroll
        for (int i = 0; i < KBW; ++i) wv[i][h] = ldg_stream16(wr + i * 16);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int64_t row = min(r0 + 8 * h + g, p.N - 1);
#pragma unroll
        for (int i = 0; i < KBW; ++i) {
            const int grp = ((kb0 + i) * 128 + c * 32) >> p.gs_shift;
            sb[i][h] = ldg_u16z(p.s + row * p.G + grp) | (ldg_u16z(p.b + row * p.G + grp) << 16);
        }
    }
    pdl_wait();  // x may be the previous kernel's output
    // Everything this thread reads from global memory after the wait is
    // issued at once: its x chunks (with the up half, or the norm weights,
    // of the prologue) and the residual of the output element it stores, so
    // that the chain after the dependency release holds one memory round
    // trip, not one per chunk.
    const bool swi = !F16 && p.pro == kRowsSwiglu, norm = !F16 && p.pro == kRowsNorm;
    uint16_t res0 = 0;  // residual of this thread's output element, first group
    if (!F16 && p.res && warp < 4) {
        const int m = 2 * c + (warp & 1);
        const int64_t n = r0 + g + 8 * (warp >> 1);
        if (m < M && n < p.N) res0 = p.res[(int64_t)m * p.res_ld + n];
    }
    constexpr int XPL = (XCH + 31) / 32;  // x chunks per lane and token
    // (long slices, KBW > 4, keep one chunk in flight at a time: their
    // registers hold the weights)
    if constexpr (XPL > 2) {
        float ss = 0.f;
        for (int q = lane; q < M * XCH; q += 32) {
            const int m = q / XCH, ck = q % XCH;
            const uint16_t *xr = p.x + (int64_t)m * p.x_ld + kb0 * 128 + ck * 8;
            uint4 v = ldg16(xr);
            if (swi) {
                const uint4 u = ldg16(xr + p.K);
                v.x = swiglu_pair(v.x, u.x);
                v.y = swiglu_pair(v.y, u.y);
                v.z = swiglu_pair(v.z, u.z);
                v.w = swiglu_pair(v.w, u.w);
            } else if (norm) {
                const uint32_t e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float lo = bf16_to_f32((uint16_t)e[t]);
                    const float hi = bf16_to_f32((uint16_t)(e[t] >> 16));
                    ss = fmaf(lo, lo, ss);
                    ss = fmaf(hi, hi, ss);
                }
            }
            const int kbi = ck >> 4, cc = (ck >> 2) & 3, i = ck & 3;
            xs[m * XCH + kbi * 16 + i * 4 + cc] = pair_permute(v);
        }
        if (norm) {
            __shared__ float ss_warp_l[16];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) ss_warp_l[warp] = ss;
            __syncthreads();
            float tot = 0.f;
            for (int w = 0; w < W; ++w) tot += ss_warp_l[w];
            const float inv = 1.0f / sqrtf(tot / (float)p.K + p.eps);
            for (int ck = lane; ck < XCH; ck += 32) {
                const int kbi = ck >> 4, cc = (ck >> 2) & 3, i = ck & 3;
                uint4 &o = xs[kbi * 16 + i * 4 + cc];
                const uint4 wn = pair_permute(ldg16(p.nw + kb0 * 128 + ck * 8));
                o.x = norm_pair(o.x, wn.x, inv);
                o.y = norm_pair(o.y, wn.y, inv);
                o.z = norm_pair(o.z, wn.z, inv);
                o.w = norm_pair(o.w, wn.w, inv);
            }
        }
    } else
    for (int m = 0; m < M; ++m) {
        // chunk ck = lane + 32 j of the slice covers codes kb0*128 + 8*ck ...
        uint4 v[XPL], u[XPL];
#pragma unroll
        for (int j = 0; j < XPL; ++j) {
            const int ck = lane + 32 * j;
            if (XCH % 32 == 0 || ck < XCH) {
                const uint16_t *xr = p.x + (int64_t)m * p.x_ld + kb0 * 128 + ck * 8;
                v[j] = ldg16(xr);
                if (swi) u[j] = ldg16(xr + p.K);  // x row = [gate (K) | up (K)]
                else if (norm) u[j] = ldg16(p.nw + kb0 * 128 + ck * 8);
            }
        }
        if (norm) {
            // (M == 1) mean of x^2 over the whole row: every warp's slice,
            // through shared memory; then each lane normalises its chunks
            __shared__ float ss_warp[16];
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < XPL; ++j) {
                if (XCH % 32 == 0 || lane + 32 * j < XCH) {
                    const uint32_t e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float lo = bf16_to_f32((uint16_t)e[t]);
                        const float hi = bf16_to_f32((uint16_t)(e[t] >> 16));
                        ss = fmaf(lo, lo, ss);
                        ss = fmaf(hi, hi, ss);
                    }
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) ss_warp[warp] = ss;
            __syncthreads();
            float tot = 0.f;
            for (int w = 0; w < W; ++w) tot += ss_warp[w];
            const float inv = 1.0f / sqrtf(tot / (float)p.K + p.eps);
#pragma unroll
            for (int j = 0; j < XPL; ++j) {
                v[j].x = norm_pair(v[j].x, u[j].x, inv);
                v[j].y = norm_pair(v[j].y, u[j].y, inv);
                v[j].z = norm_pair(v[j].z, u[j].z, inv);
                v[j].w = norm_pair(v[j].w, u[j].w, inv);
            }
        } else if (swi) {
#pragma unroll
            for (int j = 0; j < XPL; ++j) {
                v[j].x = swiglu_pair(v[j].x, u[j].x);
                v[j].y = swiglu_pair(v[j].y, u[j].y);
                v[j].z = swiglu_pair(v[j].z, u[j].z);
                v[j].w = swiglu_pair(v[j].w, u[j].w);
            }
        }
#pragma unroll
        for (int j = 0; j < XPL; ++j) {
            const int ck = lane + 32 * j;
            if (XCH % 32 == 0 || ck < XCH) {
                const int kbi = ck >> 4, cc = (ck >> 2) & 3, i = ck & 3;
                xs[m * XCH + kbi * 16 + i * 4 + cc] = pair_permute(v[j]);
            }
        }
    }
    __syncwarp();
    const uint4 *xr = xs + min(g, M - 1) * XCH + c;
#pragma unroll 1
  for (int grp2 = 0; grp2 < (PAIR ? 2 : 1); ++grp2) {
    const int64_t rg0 = r0 + 16 * grp2;  // first row of this group
    if (PAIR && grp2 == 1) {
        // the second group: its copies have landed (bounded wait); every warp
        // is done reading red for the first group's stores
        bool ok = true;
        if (!mbar_try_wait(bbar, 0)) {
            const unsigned long long t0 = global_timer_ns();
            while (!mbar_try_wait(bbar, 0)) {
                if (global_timer_ns() - t0 > kWaitLimitNs) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) {
            atomicOr(p.err, kErrWaitTimeout);
            // let the copies in flight finish (bounded) before the CTA exits
            const unsigned long long t1 = global_timer_ns();
            while (!mbar_try_wait(bbar, 0) && global_timer_ns() - t1 < kWaitLimitNs) {
            }
        }
        __syncthreads();
        if (!ok || rg0 >= p.N) return;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint8_t *wrow = bsm + (8 * h + g) * rs + kb0 * 64 + c * 16;
            const uint16_t *srow = reinterpret_cast<const uint16_t *>(bss + (8 * h + g) * p.G * 2);
            const uint16_t *brow = reinterpret_cast<const uint16_t *>(bsb + (8 * h + g) * p.G * 2);
#pragma unroll
            for (int i = 0; i < KBW; ++i) {
                wv[i][h] = *reinterpret_cast<const uint4 *>(wrow + i * 64);
                const int grp = ((kb0 + i) * 128 + c * 32) >> p.gs_shift;
                sb[i][h] = srow[grp] | ((uint32_t)brow[grp] << 16);
            }
        }
    }
    // NACC independent accumulators (short slices: 4, so that each mma waits
    // on one two steps back); summed at the end
    constexpr int NACC = (KBW == 3 || KBW == 4) ? 4 : 2;
    float acc[NACC][4] = {};
#pragma unroll
    for (int kbi = 0; kbi < KBW; ++kbi) {
        uint4 xv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[i] = xr[kbi * 16 + i * 4];
        if constexpr (F16) {
            // fp16 scales and biases: biased codes 1024 + q, exact fp16 dequant
            const Dq4h da = make_dq4h((uint16_t)sb[kbi][0], (uint16_t)(sb[kbi][0] >> 16));
            const Dq4h db = make_dq4h((uint16_t)sb[kbi][1], (uint16_t)(sb[kbi][1] >> 16));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w0 = (&wv[kbi][0].x)[i], w1 = (&wv[kbi][1].x)[i];
                const uint32_t w04 = w0 >> 4, w14 = w1 >> 4;
                const uint32_t a0 = dqh_pair(lop3_and_or(w0, 0x000F000Fu, 0x64006400u), da);
                const uint32_t a1 = dqh_pair(lop3_and_or(w1, 0x000F000Fu, 0x64006400u), db);
                const uint32_t a2 = dqh_pair(lop3_and_or(w04, 0x000F000Fu, 0x64006400u), da);
                const uint32_t a3 = dqh_pair(lop3_and_or(w14, 0x000F000Fu, 0x64006400u), db);
                const uint32_t c0 = dqh_pair(lop3_and_or(w0 >> 8, 0x000F000Fu, 0x64006400u), da);
                const uint32_t c1 = dqh_pair(lop3_and_or(w1 >> 8, 0x000F000Fu, 0x64006400u), db);
                const uint32_t c2 = dqh_pair(lop3_and_or(w04 >> 8, 0x000F000Fu, 0x64006400u), da);
                const uint32_t c3 = dqh_pair(lop3_and_or(w14 >> 8, 0x000F000Fu, 0x64006400u), db);
                mma16816h(acc[(i * 2) % NACC], a0, a1, a2, a3, xv[i].x, xv[i].y);
                mma16816h(acc[(i * 2 + 1) % NACC], c0, c1, c2, c3, xv[i].z, xv[i].w);
            }
        } else {
            Dq4 da, db;
            da.s2 = prmt(sb[kbi][0], 0u, 0x1010u);
            da.b2 = prmt(sb[kbi][0], 0u, 0x3232u);
            db.s2 = prmt(sb[kbi][1], 0u, 0x1010u);
            db.b2 = prmt(sb[kbi][1], 0u, 0x3232u);
            da.n2 = bf2_fma(da.s2, 0xC300C300u, 0x80008000u);  // exact -128*s
            db.n2 = bf2_fma(db.s2, 0xC300C300u, 0x80008000u);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w0 = (&wv[kbi][0].x)[i], w1 = (&wv[kbi][1].x)[i];
                const uint32_t w04 = w0 >> 4, w14 = w1 >> 4;
                const uint32_t a0 = dq4_pair(lop3_and_or(w0, 0x000F000Fu, 0x43004300u), da);
                const uint32_t a1 = dq4_pair(lop3_and_or(w1, 0x000F000Fu, 0x43004300u), db);
                const uint32_t a2 = dq4_pair(lop3_and_or(w04, 0x000F000Fu, 0x43004300u), da);
                const uint32_t a3 = dq4_pair(lop3_and_or(w14, 0x000F000Fu, 0x43004300u), db);
                const uint32_t c0 = dq4_pair(lop3_and_or(w0 >> 8, 0x000F000Fu, 0x43004300u), da);
                const uint32_t c1 = dq4_pair(lop3_and_or(w1 >> 8, 0x000F000Fu, 0x43004300u), db);
                const uint32_t c2 = dq4_pair(lop3_and_or(w04 >> 8, 0x000F000Fu, 0x43004300u), da);
                const uint32_t c3 = dq4_pair(lop3_and_or(w14 >> 8, 0x000F000Fu, 0x43004300u), db);
                mma16816(acc[(i * 2) % NACC], a0, a1, a2, a3, xv[i].x, xv[i].y);
                mma16816(acc[(i * 2 + 1) % NACC], c0, c1, c2, c3, xv[i].z, xv[i].w);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
        red[(warp * 4 + j) * 32 + lane] =
            NACC == 4 ? (acc[0][j] + acc[2][j]) + (acc[1][j] + acc[3][j]) : acc[0][j] + acc[1][j];
    __syncthreads();
    // warp j (< 4) sums accumulator element j over the K slices and stores it:
    // element j of lane (g, c) is token 2c + (j & 1) of row g + 8 (j >> 1)
    if (!F16 && p.epi_swiglu) {
        // the token's gate (row g, element 0) and up (row g + 8, element 2)
        // values of lanes c == 0, rounded to bf16 like the outputs of two
        // separate projections, then the SwiGLU op chain
        if (warp == 0 && c == 0 && rg0 < p.N) {
            float gv = 0.f, uv = 0.f;
            for (int w = 0; w < W; ++w) {
                gv += red[(w * 4 + 0) * 32 + lane];
                uv += red[(w * 4 + 2) * 32 + lane];
            }
            const uint32_t pr = (uint32_t)f32_to_bf16(gv) | ((uint32_t)f32_to_bf16(uv) << 16);
            p.y[(rg0 / 16) * 8 + g] = (uint16_t)swiglu_pair(pr & 0xFFFFu, pr >> 16);
        }
    } else if (warp < 4) {
        const int j = warp;
        float v = 0.f;
        for (int w = 0; w < W; ++w) v += red[(w * 4 + j) * 32 + lane];
        const int m = 2 * c + (j & 1);
        const int64_t n = rg0 + g + 8 * (j >> 1);
        if (m < M && n < p.N) {
            uint16_t out = f32_to_t16<F16>(v);
            if (!F16 && p.res) {
                const uint16_t r = grp2 == 0 ? res0 : p.res[(int64_t)m * p.res_ld + n];
                out = f32_to_bf16(bf16_to_f32(r) + bf16_to_f32(out));
            }
            p.y[(int64_t)m * p.y_ld + n] = out;
        }
    }
  }
}

// Dynamic shared memory of the row-group kernel: x staging and the K-slice
// sums, plus, for paired groups, the second group's rows, scales, biases and
// the mbarrier.
size_t rows_smem_bytes(int kbw, int W, int M, bool pair, int64_t K, int64_t G) {
    size_t b = (size_t)W * M * kbw * 16 * 16 + (size_t)W * 4 * 32 * sizeof(float);
    if (pair) {
        const int64_t rs = K / 2 + ((K / 2) % 128 == 0 ? 64 : 0);
        b += (size_t)(16 * rs + 16 * G * 2 * 2) + 16;
    }
    return b;
}

template <bool PAIR>
const void *rows_kernel_ptr(int kbw) {
    switch (kbw) {
        case 2: return (const void *)qgemv_rows_kernel<2, false, PAIR>;
        case 3: return (const void *)qgemv_rows_kernel<3, false, PAIR>;
        case 4: return (const void *)qgemv_rows_kernel<4, false, PAIR>;
        case 6: return (const void *)qgemv_rows_kernel<6, false, PAIR>;
        default: return (const void *)qgemv_rows_kernel<8, false, PAIR>;
    }
}

// CTAs of the row-group kernel that can be resident at once on this device
// (asked once per device and configuration).
int64_t rows_resident(int kbw, int W, int M, bool pair, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, int, bool, size_t>, int> cache;
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(d, kbw, W, M, pair, smem);
    auto it = cache.find(key);
    if (it == cache.end()) {
        const void *kern = pair ? rows_kernel_ptr<true>(kbw) : rows_kernel_ptr<false>(kbw);
        int n = 0;
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 32 * W, smem) != cudaSuccess)
            n = 0;
        cudaGetLastError();
        it = cache.emplace(key, n).first;
    }
    return (int64_t)it->second * sm_count();
}

struct RowsPlan {
    int kbw = 0;
    bool pair = false;
};

// k-blocks per warp (and whether a CTA takes two row groups, the second by
// bulk copies into shared memory) for the row-group kernel; kbw == 0 when it
// does not serve the problem.  The weights of every row group are fetched
// before the dependency release only if all the CTAs are resident at once,
// so plans that fit one wave come first: one group per CTA with short slices
// (more warps per row group finish the post-dependency work sooner; up to 12
// warps with slices of <= 4 k-blocks, measured best on 4096 and 3072
// columns), then any slicing of up to 16 warps, then two groups per CTA
// (measured: the decode step's 25 MB gate|up GEMV fits one wave that way).
// Shapes no plan fits in one wave: with at least 4 row groups per SM long
// slices (fewer warps, fewer partial sums), else short slices.
RowsPlan rows_plan(int64_t kb_total, int64_t row_groups, int M, int64_t K, int64_t G,
                   bool pair_ok) {
    static const int kShort[] = {2, 3, 4, 6, 8};
    static const int kLong[] = {8, 6, 4, 3, 2};
    auto fits = [&](int kbw, int64_t wmax) {
        return kb_total % kbw == 0 && kb_total / kbw >= 4 && kb_total / kbw <= wmax;
    };
    auto one_wave = [&](int kbw, bool pair) {
        const int W = (int)(kb_total / kbw);
        const int64_t ctas = pair ? (row_groups + 1) / 2 : row_groups;
        return rows_resident(kbw, W, M, pair, rows_smem_bytes(kbw, W, M, pair, K, G)) >= ctas;
    };
    for (int kbw : kShort)
        if (kbw <= 4 && fits(kbw, 12) && one_wave(kbw, false)) return {kbw, false};
    for (int kbw : kShort)
        if (fits(kbw, 16) && one_wave(kbw, false)) return {kbw, false};
    // (paired groups with 8-k-block slices exceed the 128 registers a
    // 512-thread launch allows and spill)
    if (pair_ok)
        for (int kbw : kShort)
            if (kbw < 8 && fits(kbw, 16) && one_wave(kbw, true)) return {kbw, true};
    if (row_groups >= 4 * (int64_t)sm_count()) {
        // (two groups per CTA measured slower here: 74.7 against 55-64 us for
        // the 128256 x 3072 LM head -- each CTA then computes its groups one
        // after the other in a wave-bound launch)
        for (int kbw : kLong)
            if (fits(kbw, 16)) return {kbw, false};
        return {};
    }
    for (int kbw : kShort)
        if (kbw <= 4 && fits(kbw, 12)) return {kbw, false};
    for (int kbw : kShort)
        if (fits(kbw, 16)) return {kbw, false};
    return {};
}

template <int KBW, bool F16, bool PAIR>
cudaError_t launch_rows(const RowsParams &p, int W, cudaStream_t stream) {
    const size_t smem = rows_smem_bytes(KBW, W, p.M, PAIR, p.K, p.G);
    auto kern = qgemv_rows_kernel<KBW, F16, PAIR>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.N + (PAIR ? 31 : 15)) / (PAIR ? 32 : 16)), 1, 1);
    cfg.blockDim = dim3(32 * W, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

// Checks shared by both entry points, then the kernel choice and launch.
cudaError_t launch_rows_checked(RowsParams p, const void *x, cudaStream_t stream,
                                bool f16 = false) {
    if (p.M < 1 || p.M > 8 || p.K % 128 || p.N < 1) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || p.x_ld % 8 || p.N > ((int64_t)1 << 31) * 16)
        return cudaErrorNotSupported;
    // x staged per warp: M x K bf16 per CTA in all (at most 96 KB, so that two
    // CTAs of consecutive calls still fit an SM side by side)
    if ((int64_t)p.M * p.K * 2 > 96 * 1024) return cudaErrorNotSupported;
    const int64_t kb_total = p.K / 128;
    // two row groups per CTA (the second by bulk copies): bf16 only; scale and
    // bias rows must be whole 16-byte pieces and 16-byte aligned
    const bool pair_ok = !f16 && (p.G * 2) % 16 == 0 &&
                         !((reinterpret_cast<uintptr_t>(p.s) | reinterpret_cast<uintptr_t>(p.b) |
                            reinterpret_cast<uintptr_t>(p.w)) & 15);
    const RowsPlan plan = rows_plan(kb_total, (p.N + 15) / 16, p.M, p.K, p.G, pair_ok);
    const int kbw = plan.kbw;
    if (!kbw) return cudaErrorNotSupported;
    const int W = (int)(kb_total / kbw);
    if (f16) {
        if (p.pro != kRowsPlain || p.res) return cudaErrorNotSupported;
        switch (kbw) {
            case 2: return launch_rows<2, true, false>(p, W, stream);
            case 3: return launch_rows<3, true, false>(p, W, stream);
            case 4: return launch_rows<4, true, false>(p, W, stream);
            case 6: return launch_rows<6, true, false>(p, W, stream);
            default: return launch_rows<8, true, false>(p, W, stream);
        }
    }
    if (plan.pair) {
        switch (kbw) {
            case 2: return launch_rows<2, false, true>(p, W, stream);
            case 3: return launch_rows<3, false, true>(p, W, stream);
            case 4: return launch_rows<4, false, true>(p, W, stream);
            case 6: return launch_rows<6, false, true>(p, W, stream);
            default: return launch_rows<8, false, true>(p, W, stream);
        }
    }
    switch (kbw) {
        case 2: return launch_rows<2, false, false>(p, W, stream);
        case 3: return launch_rows<3, false, false>(p, W, stream);
        case 4: return launch_rows<4, false, false>(p, W, stream);
        case 6: return launch_rows<6, false, false>(p, W, stream);
        default: return launch_rows<8, false, false>(p, W, stream);
    }
}

RowsParams rows_params(const uint32_t *w, const uint16_t *s, const uint16_t *b, int64_t N,
                       int64_t K, int gs, const uint16_t *x, int64_t x_ld, int M, uint16_t *y,
                       int64_t y_ld) {
    RowsParams p;
    p.w = w;
    p.s = s;
    p.b = b;
    p.x = x;
    p.y = y;
    p.N = N;
    p.K = K;
    p.Kw = K / 8;
    p.G = K / gs;
    p.x_ld = x_ld;
    p.y_ld = y_ld;
    p.gs_shift = gs == 32 ? 5 : (gs == 64 ? 6 : 7);
    p.M = M;
    p.pro = kRowsPlain;
    p.nw = nullptr;
    p.eps = 0.f;
    p.res = nullptr;
    p.res_ld = 0;
    p.err = device_error_word();
    p.epi_swiglu = 0;
    return p;
}

// The row-group kernel serves q when q is one plain problem of at most 8
// tokens with 4-bit codes, K a multiple of 128 that splits into 4..16 warps,
// and x rows 16-byte aligned; returns cudaErrorNotSupported otherwise.
cudaError_t try_launch_rows(const GemvProblems &q, cudaStream_t stream) {
    const bool plain = q.P == 1 && !q.expert && !q.expert_is_p && !q.m_count && !q.m_offset &&
                       !q.x_rows && !q.lhs && !q.y_rows && q.x_div == 0 && !q.w2 && !q.push &&
                       !q.out_f32 && !q.swiglu;
    if (!plain || q.bits != 4) return cudaErrorNotSupported;
    return launch_rows_checked(rows_params(q.w, q.s, q.b, q.N, q.K, q.gs, q.x, q.x_ld, q.M,
                                           static_cast<uint16_t *>(q.y), q.y_ld),
                               q.x, stream);
}

}  // namespace

bool rows_fused_supported(int64_t N, int64_t K, int bits) {
    return bits == 4 && N >= 1 && K % 128 == 0 && K * 2 <= 96 * 1024 &&
           N <= ((int64_t)1 << 31) * 16 && rows_plan(K / 128, (N + 15) / 16, 1, K, K / 64, false).kbw != 0;
}

cudaError_t launch_rows_f16(const uint16_t *x, int M, const uint32_t *w, const uint16_t *s,
                            const uint16_t *b, int64_t N, int64_t K, int bits, int gs, uint16_t *y,
                            cudaStream_t stream) {
    if (bits != 4) return cudaErrorNotSupported;
    return launch_rows_checked(rows_params(w, s, b, N, K, gs, x, K, M, y, N), x, stream, true);
}

cudaError_t launch_rows_fused(const RowsFusedArgs &a, cudaStream_t stream) {
    if (a.bits != 4) return cudaErrorNotSupported;
    if (a.prologue != kRowsPlain && a.M != 1) return cudaErrorNotSupported;
    if (a.prologue == kRowsSwiglu && (a.x_ld < 2 * a.K)) return cudaErrorNotSupported;
    if (a.prologue == kRowsNorm && (!a.norm_w || (reinterpret_cast<uintptr_t>(a.norm_w) & 15)))
        return cudaErrorNotSupported;
    if (a.epi_swiglu && (a.M != 1 || a.N % 16 || a.res)) return cudaErrorNotSupported;
    RowsParams p = rows_params(a.w, a.s, a.b, a.N, a.K, a.gs, a.x, a.x_ld, a.M, a.y, a.y_ld);
    p.epi_swiglu = a.epi_swiglu;
    p.pro = a.prologue;
    p.nw = a.norm_w;
    p.eps = a.eps;
    p.res = a.res;
    p.res_ld = a.res_ld;
    return launch_rows_checked(p, a.x, stream);
}

const char *gemv_push_unsupported(const GemvProblems &q) {
    // the output fan-out lives in the TMA-fed kernel: its conditions, below
    const uintptr_t sb_bits = reinterpret_cast<uintptr_t>(q.s) | reinterpret_cast<uintptr_t>(q.b) |
                              reinterpret_cast<uintptr_t>(q.s2 ? q.s2 : q.s) |
                              reinterpret_cast<uintptr_t>(q.b2 ? q.b2 : q.b);
    if (q.K % 256) return "K must be a multiple of 256 for M <= 32";
    if (q.bits == 8 && q.gs == 128) return "8-bit codes with group size 128 are not served for M <= 32";
    if ((reinterpret_cast<uintptr_t>(q.x) & 15) || q.x_ld % 8)
        return "x rows must be 16-byte aligned";
    if (sb_bits & 15) return "scales and biases must be 16-byte aligned for M <= 32";
    return nullptr;  // (and the driver must provide tensor maps: tensor_maps_available())
}

cudaError_t launch_gemv(const GemvProblems &q, cudaStream_t stream) {
    {
        const cudaError_t e = try_launch_rows(q, stream);
        if (e != cudaErrorNotSupported) return e;
    }
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
    prm.x_div = q.x_div;
    prm.y_rows = q.y_rows;
    prm.expert_is_p = q.expert_is_p ? 1 : 0;
    prm.x_from_offset = q.x_from_offset ? 1 : 0;
    prm.y = q.y;
    prm.y_ld = q.y_ld;
    prm.out_f32 = q.out_f32;
    prm.swiglu = q.swiglu;
    prm.kb_total = (int)((prm.Kw + 15) / 16);
    prm.kb_full = (int)(prm.Kw / 16);
    prm.err = device_error_word();
    if (q.push) prm.push = *q.push;

    const bool dual = q.w2 != nullptr;
    const int max_m = std::max(1, q.max_m);
    const int size_m = q.tile_m > 0 ? std::min(q.tile_m, max_m) : max_m;
    const int nt = size_m <= 8 ? 1 : (size_m <= 16 ? 2 : 4);

    // ---- asynchronously fed kernel (the default).  Its scale/bias spans are
    // 4-16 byte cp.async copies: pointers aligned to less than 16 bytes (a
    // legal bf16 sub-view) take the register-fed kernel, which reads them by
    // element.
    const uintptr_t sb_bits = reinterpret_cast<uintptr_t>(q.s) | reinterpret_cast<uintptr_t>(q.b) |
                              reinterpret_cast<uintptr_t>(prm.s2) |
                              reinterpret_cast<uintptr_t>(prm.b2);
    if (q.K % 256 == 0 && !(q.bits == 8 && q.gs == 128) &&
        (reinterpret_cast<uintptr_t>(q.x) & 15) == 0 && q.x_ld % 8 == 0 && (sb_bits & 15) == 0) {
        // 32 rows per consumer warp (shares the activation work between two
        // row tiles) unless that leaves fewer than ~2 CTAs per SM
        const int rt_t = (!dual && nt == 1 && ((q.N + 127) / 128) * (int64_t)q.P >= 2 * sm_count())
                             ? 2
                             : 1;
        const int rows_cta = kTConsumers * 16 * rt_t;
        CUtensorMap m1, m2;
        const uint64_t rows = (uint64_t)q.E * (uint64_t)q.N;
        bool ok = make_map_2d(&m1, CU_TENSOR_MAP_DATA_TYPE_UINT32, q.w, (uint64_t)prm.Kw, rows,
                              (uint64_t)prm.Kw * 4, kTStageWords, rows_cta,
                              CU_TENSOR_MAP_SWIZZLE_128B);
        if (ok)
            ok = make_map_2d(&m2, CU_TENSOR_MAP_DATA_TYPE_UINT32, dual ? q.w2 : q.w,
                             (uint64_t)prm.Kw, rows, (uint64_t)prm.Kw * 4, kTStageWords,
                             rows_cta, CU_TENSOR_MAP_SWIZZLE_128B);
        if (ok) {
            const int64_t row_blocks = (q.N + rows_cta - 1) / rows_cta;
            const int64_t tasks = row_blocks * (int64_t)q.P;
            const int n_stg = (int)(q.K / (kTStageWords * 32 / q.bits));
            prm.mx = std::min(max_m, 8 * nt);
            // Split K over a cluster until there are ~4 CTAs of work per SM,
            // keeping >= 2 stages per CTA.  Only single-pass problems (every
            // problem's tokens fit one pass) may split: see the kernel.
            const int64_t target = (int64_t)sm_count() * 4;
            int ksplit = 1;
            const int kmax = max_m > 1 ? 4 : 8;  // measured: deeper splits only pay at M = 1
            if (max_m <= prm.mx)
                while (ksplit < kmax && tasks * ksplit < target && n_stg >= 4 * ksplit) ksplit <<= 1;
            prm.s_cta = 1;
            dim3 grid((unsigned)row_blocks, (unsigned)ksplit, (unsigned)q.P);
            if (q.bits == 4)
                return dual ? dispatch_tma<4, true>(m1, m2, prm, nt, rt_t, grid, ksplit, stream)
                            : dispatch_tma<4, false>(m1, m2, prm, nt, rt_t, grid, ksplit, stream);
            return dual ? dispatch_tma<8, true>(m1, m2, prm, nt, rt_t, grid, ksplit, stream)
                        : dispatch_tma<8, false>(m1, m2, prm, nt, rt_t, grid, ksplit, stream);
        }
    }

    // ---- register-fed kernel (when no tensor map can be encoded)
    if (q.push) return cudaErrorNotSupported;  // the output fan-out is in the TMA-fed kernel only
    const int rt = (!dual && nt == 1 && q.N >= 64) ? 2 : 1;
    const int64_t row_groups = (q.N + 16 * rt - 1) / (16 * rt);
    const int64_t tasks = row_groups * (int64_t)q.P;
    // Split K until there are ~16 warps of work per SM, keeping >= 2 k-blocks
    // per warp (the register double buffer) and at most 8 CTAs per cluster.
    const int64_t target = (int64_t)sm_count() * 16;
    int ksplit = 1;
    while (ksplit < 32 && tasks * ksplit < target && prm.kb_total >= ksplit * 4) ksplit <<= 1;
    const int s_cta = std::min(ksplit, 4);
    const int cluster = ksplit / s_cta;
    prm.s_cta = s_cta;
    const int groups_per_cta = 4 / s_cta;
    dim3 grid((unsigned)((row_groups + groups_per_cta - 1) / groups_per_cta), (unsigned)cluster,
              (unsigned)q.P);
    if (q.bits == 4)
        return dual ? dispatch<4, true>(prm, nt, rt, grid, cluster, stream)
                    : dispatch<4, false>(prm, nt, rt, grid, cluster, stream);
    return dual ? dispatch<8, true>(prm, nt, rt, grid, cluster, stream)
                : dispatch<8, false>(prm, nt, rt, grid, cluster, stream);
}

}  // namespace nq
