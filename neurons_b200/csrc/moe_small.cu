// moe_small.cu -- the MoE switch step for a few tokens (every (token, slot)
// pair its own problem, T * top_k <= E), in two kernels instead of three:
//
//   up:   h[p] = bf16(silu(x[t] . Wg[e_p]^T) * (x[t] . Wu[e_p]^T)),  p = t * k + j
//   down: y[t] = bf16(sum_j bf16(score_tj) * (h[p] . Wd[e_p]^T))  (slot order)
//
// (qwen3_transformer_moe_model_mlx.cpp:29-79; the rounding points of the
// batched switch step, nq_moe_switch.)  Both follow the row-group decode
// GEMV: a CTA owns 16 weight rows and all of K, every lane loads its whole
// share of the weights at once, and the dequantization into mma.sync A
// fragments is the exact one of the other kernels.
//   * The up kernel waits for the routing (the previous kernel), then loads the
//     gate and up rows of its pair's expert and the token's x.
//   * The down kernel owns 16 output rows of one token over all k of its
//     pairs, so it forms the score-weighted sum itself -- no fp32 d round trip
//     and no combine launch.  The up kernel signals its dependents only after
//     its own dependency wait, so by the time the down kernel starts, the
//     routing (two kernels back) is complete: the down kernel reads it and
//     loads all k experts' weight rows before its own wait, under the up
//     kernel, and waits only for h.
#include <cuda_runtime.h>

#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

constexpr int kUpKbw = 2;     // k-blocks (128 codes) per warp, up kernel
constexpr int kMaxSlots = 8;  // top_k served by the down kernel

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ld_u16z(const uint16_t *p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// One warp's slice of a bf16 row into shared memory, pairs permuted to the
// order of the mma.sync B fragments ((x0,x4),(x1,x5),(x2,x6),(x3,x7)) and
// chunks laid out so that the four lanes of a row read consecutive chunks.
template <int KBW>
__device__ __forceinline__ void stage_slice(const uint16_t *row, int kb0, int lane, uint4 *xs) {
    constexpr int XCH = KBW * 16;
    for (int ck = lane; ck < XCH; ck += 32) {
        const uint4 v = *reinterpret_cast<const uint4 *>(row + kb0 * 128 + ck * 8);
        uint4 o;
        o.x = prmt(v.x, v.z, 0x5410u);
        o.y = prmt(v.x, v.z, 0x7632u);
        o.z = prmt(v.y, v.w, 0x5410u);
        o.w = prmt(v.y, v.w, 0x7632u);
        const int kbi = ck >> 4, cc = (ck >> 2) & 3, i = ck & 3;
        xs[kbi * 16 + i * 4 + cc] = o;
    }
}

// acc += dequant(w rows g, g+8; this warp's k-blocks) . x-slice fragments
template <int KBW>
__device__ __forceinline__ void dq_mma(float (&acc)[2][4], const uint4 (&wv)[KBW][2],
                                       const uint32_t (&sv)[KBW][2], const uint32_t (&bv)[KBW][2],
                                       const uint4 *xr) {
#pragma unroll
    for (int kbi = 0; kbi < KBW; ++kbi) {
        uint4 xv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[i] = xr[kbi * 16 + i * 4];
        Dq4 da, db;
        da.s2 = prmt(sv[kbi][0], 0u, 0x1010u);
        da.b2 = prmt(bv[kbi][0], 0u, 0x1010u);
        db.s2 = prmt(sv[kbi][1], 0u, 0x1010u);
        db.b2 = prmt(bv[kbi][1], 0u, 0x1010u);
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
            mma_bf16(acc[0], a0, a1, a2, a3, xv[i].x, xv[i].y);
            mma_bf16(acc[1], c0, c1, c2, c3, xv[i].z, xv[i].w);
        }
    }
}

// This lane's weight share of rows (row_g, row_g + 8) of a [*, K] packed
// matrix: k-blocks [kb0, kb0 + KBW), 16 bytes per row per k-block, and the
// matching scales and biases.
template <int KBW>
__device__ __forceinline__ void load_rows(const uint32_t *w, const uint16_t *s, const uint16_t *b,
                                          int64_t row_g, int64_t Kw, int64_t G, int gs_shift,
                                          int kb0, int c, uint4 (&wv)[KBW][2],
                                          uint32_t (&sv)[KBW][2], uint32_t (&bv)[KBW][2]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int64_t row = row_g + 8 * h;
#pragma unroll
        for (int i = 0; i < KBW; ++i) {
            wv[i][h] = ld_stream16(w + row * Kw + (kb0 + i) * 16 + 4 * c);
            const int grp = ((kb0 + i) * 128 + c * 32) >> gs_shift;
            sv[i][h] = ld_u16z(s + row * G + grp);
            bv[i][h] = ld_u16z(b + row * G + grp);
        }
    }
}

struct SmallArgs {
    const uint16_t *x;                 // [T, H]
    const int32_t *idx;                // [T, k]
    const float *scores;               // [T, k]
    const uint32_t *gw, *uw, *dw;      // [E, I, H/8], [E, I, H/8], [E, H, I/8]
    const uint16_t *gs, *gb, *us, *ub, *ds, *db;
    uint16_t *h;                       // [T*k, I]
    uint16_t *y;                       // [T, H]
    unsigned int *err;
    int64_t H, I;
    int E, top_k, gs_shift;
};

// grid (I / 16, T * k); W = H / (128 * kUpKbw) warps.  80 registers (87
// uncapped) let three 256-thread CTAs share an SM, so the T = 1 grid at the
// Qwen3 dims (48 x 8 CTAs) is one wave: measured 21.4 -> 20.7 us per step.
__global__ void __maxnreg__(80) moe_small_up_kernel(const SmallArgs a) {
    constexpr int KBW = kUpKbw, XCH = KBW * 16;
    extern __shared__ __align__(16) uint4 up_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    pdl_wait();                // the routing comes from the previous kernel
    pdl_launch_dependents();   // after the wait: see the file comment
    const int64_t p = blockIdx.y, t = p / a.top_k;
    const int e = a.idx[p];
    const int64_t r0 = (int64_t)blockIdx.x * 16;
    if (e < 0 || e >= a.E) {   // uniform over the CTA
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, kErrBadIndex);
        if (threadIdx.x < 16) a.h[p * a.I + r0 + threadIdx.x] = 0;
        return;
    }
    const int kb0 = warp * KBW;
    const int64_t Kw = a.H / 8, G = a.H >> a.gs_shift;
    uint4 wg[KBW][2], wu[KBW][2];
    uint32_t sg[KBW][2], bg[KBW][2], su[KBW][2], bu[KBW][2];
    const int64_t row_g = (int64_t)e * a.I + r0 + g;
    load_rows<KBW>(a.gw, a.gs, a.gb, row_g, Kw, G, a.gs_shift, kb0, c, wg, sg, bg);
    load_rows<KBW>(a.uw, a.us, a.ub, row_g, Kw, G, a.gs_shift, kb0, c, wu, su, bu);
    uint4 *xs = up_smem + (size_t)warp * XCH;
    stage_slice<KBW>(a.x + t * a.H, kb0, lane, xs);
    __syncwarp();
    float ag[2][4] = {}, au[2][4] = {};
    dq_mma<KBW>(ag, wg, sg, bg, xs + c);
    dq_mma<KBW>(au, wu, su, bu, xs + c);
    float *red = reinterpret_cast<float *>(up_smem + (size_t)W * XCH);  // [W][8][32]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        red[(warp * 8 + j) * 32 + lane] = ag[0][j] + ag[1][j];
        red[(warp * 8 + 4 + j) * 32 + lane] = au[0][j] + au[1][j];
    }
    __syncthreads();
    // element j of lane (g, c) is token 2c + (j & 1) of row g + 8 (j >> 1):
    // the one token is element 0 (row g) and 2 (row g + 8) of the c == 0 lanes
    if (warp < 2 && c == 0) {
        const int j = 2 * warp;
        float gv = 0.f, uv = 0.f;
        for (int w = 0; w < W; ++w) {
            gv += red[(w * 8 + j) * 32 + lane];
            uv += red[(w * 8 + 4 + j) * 32 + lane];
        }
        a.h[p * a.I + r0 + g + 8 * warp] = f32_to_bf16(silu_f32(gv) * uv);
    }
}

// grid (H / 16, T); W = I / (128 * KBW) warps (4..8); top_k <= kMaxSlots
template <int KBW>
__global__ void __launch_bounds__(256) moe_small_down_kernel(const SmallArgs a) {
    constexpr int XCH = KBW * 16;
    extern __shared__ __align__(16) uint4 dn_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    pdl_launch_dependents();
    const int64_t t = blockIdx.y, r0 = (int64_t)blockIdx.x * 16;
    const int k = a.top_k, kb0 = warp * KBW;
    const int64_t Kw = a.I / 8, G = a.I >> a.gs_shift;
    // The routing is complete here (the up kernel signalled after its own
    // wait): every slot's expert rows load before this kernel's wait.
    uint4 wd[kMaxSlots][KBW][2];
    uint32_t sd[kMaxSlots][KBW][2], bd[kMaxSlots][KBW][2];
    unsigned valid = 0;
#pragma unroll
    for (int j = 0; j < kMaxSlots; ++j) {
        if (j < k) {
            const int e = a.idx[t * k + j];
            if (e >= 0 && e < a.E) {
                valid |= 1u << j;
                load_rows<KBW>(a.dw, a.ds, a.db, (int64_t)e * a.H + r0 + g, Kw, G, a.gs_shift,
                               kb0, c, wd[j], sd[j], bd[j]);
            }
        }
    }
    pdl_wait();  // h comes from the up kernel
    uint4 *xs = dn_smem + (size_t)warp * kMaxSlots * XCH;  // [slot][XCH] per warp
#pragma unroll
    for (int j = 0; j < kMaxSlots; ++j)
        if ((valid >> j) & 1u) stage_slice<KBW>(a.h + (t * k + j) * a.I, kb0, lane, xs + j * XCH);
    __syncwarp();
    float *red = reinterpret_cast<float *>(dn_smem + (size_t)W * kMaxSlots * XCH);  // [W][k][2][32]
#pragma unroll
    for (int j = 0; j < kMaxSlots; ++j) {
        if ((valid >> j) & 1u) {
            float acc[2][4] = {};
            dq_mma<KBW>(acc, wd[j], sd[j], bd[j], xs + j * XCH + c);
            // the token's elements: 0 (row g) and 2 (row g + 8) of the c == 0 lanes
            red[((warp * kMaxSlots + j) * 2 + 0) * 32 + lane] = acc[0][0] + acc[1][0];
            red[((warp * kMaxSlots + j) * 2 + 1) * 32 + lane] = acc[0][2] + acc[1][2];
        }
    }
    __syncthreads();
    if (warp < 2 && c == 0) {
        // y = sum over the slots in slot order of bf16(score) * d, d the fp32
        // row sum over the K slices (as the combine kernel forms it)
        float v = 0.f;
        for (int j = 0; j < k; ++j) {
            if (!((valid >> j) & 1u)) continue;
            float d = 0.f;
            for (int w = 0; w < W; ++w) d += red[((w * kMaxSlots + j) * 2 + warp) * 32 + lane];
            const float sc = bf16_to_f32(f32_to_bf16(a.scores[t * k + j]));
            v = __fmaf_rn(sc, d, v);
        }
        a.y[t * a.H + r0 + g + 8 * warp] = f32_to_bf16(v);
    }
}

template <typename... Args>
cudaError_t launch_small(void (*kern)(Args...), dim3 grid, unsigned threads, size_t smem,
                         cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace

bool moe_small_supported(int64_t T, int64_t H, int64_t I, int64_t E, int64_t top_k, int bits,
                         const void *x) {
    if (bits != 4 || T < 1 || T * top_k > E || top_k > kMaxSlots) return false;
    if (H % (128 * kUpKbw) || H / (128 * kUpKbw) < 4 || H / (128 * kUpKbw) > 16) return false;
    if (H % 16 || I % 16) return false;
    // down kernel: 4..8 warps of 1 k-block (I = 512..1024) or of 2 (I = 1280..2048)
    const int64_t kb = I / 128;
    if (I % 128 || kb < 4 || kb > 16 || (kb > 8 && kb % 2)) return false;
    return (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

cudaError_t launch_moe_small(const uint16_t *x, int64_t T, int64_t H, int64_t I, int64_t E,
                             int64_t top_k, const int32_t *idx, const float *scores,
                             const uint32_t *gw, const uint16_t *gs, const uint16_t *gb,
                             const uint32_t *uw, const uint16_t *us, const uint16_t *ub,
                             const uint32_t *dw, const uint16_t *ds, const uint16_t *db, int gsz,
                             uint16_t *h, uint16_t *y, cudaStream_t stream) {
    SmallArgs a;
    a.x = x; a.idx = idx; a.scores = scores;
    a.gw = gw; a.gs = gs; a.gb = gb;
    a.uw = uw; a.us = us; a.ub = ub;
    a.dw = dw; a.ds = ds; a.db = db;
    a.h = h; a.y = y;
    a.err = device_error_word();
    a.H = H; a.I = I; a.E = (int)E; a.top_k = (int)top_k;
    a.gs_shift = gsz == 32 ? 5 : (gsz == 64 ? 6 : 7);
    const int Wu = (int)(H / (128 * kUpKbw));
    const size_t up_smem = (size_t)Wu * kUpKbw * 16 * 16 + (size_t)Wu * 8 * 32 * sizeof(float);
    cudaError_t e = launch_small(moe_small_up_kernel, dim3((unsigned)(I / 16), (unsigned)(T * top_k)),
                                 32u * Wu, up_smem, stream, (const SmallArgs)a);
    if (e != cudaSuccess) return e;
    const int64_t kb = I / 128;
    const int kbw = kb <= 8 ? 1 : 2;
    const int Wd = (int)(kb / kbw);
    const size_t dn_smem = (size_t)Wd * kMaxSlots * kbw * 16 * 16 +
                           (size_t)Wd * kMaxSlots * 2 * 32 * sizeof(float);
    auto dk = kbw == 1 ? moe_small_down_kernel<1> : moe_small_down_kernel<2>;
    if (dn_smem > 48 * 1024 &&
        (e = cudaFuncSetAttribute(dk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)dn_smem)) != cudaSuccess)
        return e;
    return launch_small(dk, dim3((unsigned)(H / 16), (unsigned)T), 32u * Wd, dn_smem, stream,
                        (const SmallArgs)a);
}

}  // namespace nq
