// gemm_tc_moe.cu -- the expert-grouped quantized GEMMs of the MoE switch step
// on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Restates the gather_qmm calls of the switch step
// (compute/src/compute/model/qwen3_transformer_moe_model_mlx.cpp:69-74 and
// qwen3_moe_model_mlx.cpp:356-363) for a whole batch of tokens at once.  The
// (token, slot) pairs are sorted by expert into "grouped order" g (moe.cu);
// a tile is (expert e, first grouped row g0, count <= 256), built on the
// device.  One CTA multiplies one weight-row block of expert e with one tile:
//
//   up kernel:    h[g, n] = bf16( silu(x[tok(g)] . Wg[e, n]) * (x[tok(g)] . Wu[e, n]) )
//                 The 128-row weight tile holds 64 gate rows (TMEM lanes
//                 0-63) and the same 64 rows of up (lanes 64-127), so one
//                 accumulator holds both factors of every h element.  Token
//                 rows come from xg, x copied into grouped order (moe.cu).
//   down kernel:  d[pair(g), n] = h[g] . Wd[e, n]   (fp32)
// Both kernels read their token rows (xg or h, contiguous per expert) with one
// TMA box of 256 rows x 64 bf16 per stage, 128-byte swizzled.
//
// The MMA's N is the tile's count rounded up to 16 (a tile wastes at most 15
// token columns).  Roles as in the dense kernel (gemm_tc.cu): warps 0-15 turn
// the packed codes into exact MLX bf16 values and store them into TMEM (the
// MMA's A operand), warp 16 loads, warp 17 allocates TMEM and issues the
// MMAs.  Every wait is bounded; on a timeout the CTA raises the device error
// word, drains and frees its TMEM.
#include <cuda.h>

#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

constexpr int kBlockW = 128;       // weight rows per CTA (UMMA M)
constexpr int kBlockK = 64;        // codes per stage
constexpr int kMaxTok = kMoeTileTokens;
constexpr int kSbAhead = 2;       // scale/bias prefetch depth, in this warp's iterations
constexpr int kStageArrivals = 8;  // dequant warps working on one stage
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;
constexpr int kThreads = 576;
constexpr int kXchgBytes = 8 * 2 * 16 * 32 * 4;  // up epilogue: 8 warp pairs x 2 buffers

template <int BITS>
struct MoeCfg {
    static constexpr int kXStageBytes = kMaxTok * kBlockK * 2;
    static constexpr int kWStageBytes = kBlockW * kBlockK * BITS / 8;
    static constexpr int kStageBytes = kXStageBytes + kWStageBytes;
    static constexpr int kStages = BITS == 4 ? 6 : 5;
    static constexpr int kACol0 = kMaxTok;  // accumulator: columns [0, 256)
    static constexpr int kTmemCols = 512;
    static_assert(kACol0 + kStages * 32 <= kTmemCols, "TMEM budget");
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256 + kMaxTok * 4;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    // epilogue exchange of the up kernel: 8 warp pairs x 2 buffers x [16][32] fp32
    static_assert(kXchgBytes + kMaxTok * 128 <= kStages * kXStageBytes, "exchange + h staging");
};

struct MoeTcParams {
    int64_t N, K, G;                  // weight rows per expert, reduction length, groups per row
    int gs_shift, num_kb;
    const uint16_t *s, *b;            // [E, N, G] (gate for the up kernel)
    const uint16_t *s2, *b2;          // up (up kernel only)
    const int4 *tiles;                // {expert, g0, count, 0}
    const int32_t *n_tiles;
    const int32_t *rows;              // down: pair of grouped row
    void *y;                          // up: h [P, N] bf16 (grouped rows); down: d [P, N] fp32
    int64_t y_ld;
    int h_map;                        // up: h leaves through tmap_h (16-row TMA stores)
    unsigned int *err;
    // down, fused combine (fuse != 0): the last of a token's routed pairs to
    // land in an n-block sums them (see the epilogue)
    int fuse;
    const int32_t *idx;               // [T, top_k] routing
    const float *scores;              // [T, top_k]
    int top_k, e0, ne;                // this call's experts [e0, e0 + ne)
    int32_t *cnt;                     // [T, n-blocks] arrivals, zero at the start of the call
    uint16_t *out;                    // y [T, N] bf16 (when ro.n == 0)
    MoeRowsOut ro;                    // fp32 rows into other ranks' buffers (ro.n > 0)
};

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

template <int BITS, bool UP>
__global__ void __launch_bounds__(kThreads, 1)
    tc_moe_kernel(const __grid_constant__ CUtensorMap tmap_w1,
                  const __grid_constant__ CUtensorMap tmap_w2,
                  const __grid_constant__ CUtensorMap tmap_x,
                  const __grid_constant__ CUtensorMap tmap_h, const MoeTcParams prm) {
    using Cfg = MoeCfg<BITS>;
    constexpr int S = Cfg::kStages;
    if ((int)blockIdx.y >= *prm.n_tiles) return;  // uniform: beyond the tile list
    const int4 tile = prm.tiles[blockIdx.y];
    const int e = tile.x, g0 = tile.y, cnt = tile.z;
    const int n_mma = (cnt + 15) & ~15;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint8_t *xs = smem;                          // S x [256][128 B] tokens
    uint8_t *ws = smem + S * Cfg::kXStageBytes;  // S x [128][32|64 B] codes
    uint64_t *bars = reinterpret_cast<uint64_t *>(ws + S * Cfg::kWStageBytes);
    uint64_t *full = bars;
    uint64_t *empty = bars + S;
    uint64_t *afull = bars + 2 * S;
    uint64_t *accfull = bars + 3 * S;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 3 * S + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_holder + 1);
    int32_t *rows = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(bars) + 256);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t nb = blockIdx.x;
    const int64_t nbase = nb * (UP ? kBlockW / 2 : kBlockW);  // first weight row of the block
    const int32_t wrow0 = (int32_t)((int64_t)e * prm.N + nbase);
    const int num_kb = prm.num_kb;

    if (!UP && threadIdx.x < kMaxTok) {
        const int t = threadIdx.x;
        rows[t] = t < cnt ? prm.rows[g0 + t] : 0;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);  // TMA bytes of the stage landed
            mbar_init(&empty[s], 1 + kStageArrivals);
            mbar_init(&afull[s], kStageArrivals);
        }
        mbar_init(accfull, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == kProducerWarp && lane == 0) {
        prefetch_tmap(&tmap_w1);
        if (UP) prefetch_tmap(&tmap_w2);
        prefetch_tmap(&tmap_x);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_holder, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            constexpr int kWords = kBlockK * BITS / 32;
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % S;
                const uint32_t ph = (uint32_t)(kb / S) & 1u;
                if (!mbar_wait_or_abort(&empty[s], ph ^ 1u, abort, prm.err)) break;
                mbar_expect_tx(&full[s], Cfg::kXStageBytes + Cfg::kWStageBytes);
                tma_load_2d(xs + s * Cfg::kXStageBytes, &tmap_x, &full[s], kb * kBlockK, g0);
                uint8_t *wst = ws + s * Cfg::kWStageBytes;
                tma_load_2d(wst, &tmap_w1, &full[s], kb * kWords, wrow0);
                if (UP)  // the up rows fill the second half of the weight tile
                    tma_load_2d(wst + Cfg::kWStageBytes / 2, &tmap_w2, &full[s], kb * kWords, wrow0);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(kBlockW, n_mma);
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % S;
                const uint32_t ph = (uint32_t)(kb / S) & 1u;
                if (!mbar_wait_or_abort(&full[s], ph, abort, prm.err)) break;
                if (!mbar_wait_or_abort(&afull[s], ph, abort, prm.err)) break;
                tc_fence_after();
                const uint64_t bdesc = smem_desc_k_sw128(smem_u32(xs + s * Cfg::kXStageBytes));
#pragma unroll
                for (int j = 0; j < kBlockK / 16; ++j) {
                    const uint32_t a_tmem = tmem_base + (uint32_t)(Cfg::kACol0 + s * 32 + j * 8);
                    umma_ts(tmem_base, a_tmem, bdesc + (uint64_t)(j * 2), idesc,
                            (kb > 0 || j > 0) ? 1u : 0u);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(accfull);
        }
    } else {
        // ------------------------------------------------ dequantizers
        const int q = warp & 3;          // TMEM lane quadrant
        const int h = (warp >> 2) & 1;   // which 32 codes of the stage
        const int par = warp >> 3;       // stages kb % 2 == par
        const int r = q * 32 + lane;     // row of the 128-row tile
        const bool second = UP && r >= 64;
        const int64_t nrow = nbase + (UP ? (r & 63) : r);  // row inside expert e
        const bool row_ok = nrow < prm.N;
        const int64_t srow_off = ((int64_t)e * prm.N + (row_ok ? nrow : 0)) * prm.G;
        const uint16_t *srow = (second ? prm.s2 : prm.s) + srow_off;
        const uint16_t *brow = (second ? prm.b2 : prm.b) + srow_off;
        auto load_sb = [&](int kb, uint16_t &sv, uint16_t &bv) {
            const int k = kb * kBlockK + 32 * h;
            sv = 0;
            bv = 0;
            if (row_ok && kb < num_kb) {
                sv = srow[k >> prm.gs_shift];
                bv = brow[k >> prm.gs_shift];
            }
        };
        // Scale and bias of this thread's row for its next kSbAhead stages, in
        // a shift register: the load for a stage is issued kSbAhead of this
        // warp's iterations before its use, which covers an HBM round trip.
        uint16_t sq[kSbAhead], bq[kSbAhead];
#pragma unroll
        for (int i = 0; i < kSbAhead; ++i) load_sb(par + 2 * i, sq[i], bq[i]);
        const uint32_t t_lane = (uint32_t)(q * 32) << 16;
        for (int kb = par; kb < num_kb; kb += 2) {
            const int s = kb % S;
            const uint32_t ph = (uint32_t)(kb / S) & 1u;
            if (!mbar_wait_or_abort(&full[s], ph, abort, prm.err)) break;
            tc_fence_after();
            uint32_t out[16];
            const uint8_t *wst = ws + s * Cfg::kWStageBytes;
            if constexpr (BITS == 4) {
                const uint4 v = *reinterpret_cast<const uint4 *>(
                    wst + r * 32 + 16 * (h ^ ((r >> 2) & 1)));
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                const Dq4 d = make_dq4(sq[0], bq[0]);
                const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t d0 = dq4_pair(q4_pair_biased(words[i], 0), d);
                    const uint32_t d1 = dq4_pair(q4_pair_biased(words[i], 1), d);
                    const uint32_t d2 = dq4_pair(q4_pair_biased(words[i], 2), d);
                    const uint32_t d3 = dq4_pair(q4_pair_biased(words[i], 3), d);
                    out[4 * i + 0] = prmt(d0, d1, 0x5410u);
                    out[4 * i + 1] = prmt(d2, d3, 0x5410u);
                    out[4 * i + 2] = prmt(d0, d1, 0x7632u);
                    out[4 * i + 3] = prmt(d2, d3, 0x7632u);
                }
            } else {
                const int x = (r >> 1) & 3;
                const uint4 v0 = *reinterpret_cast<const uint4 *>(wst + r * 64 + 16 * ((2 * h) ^ x));
                const uint4 v1 =
                    *reinterpret_cast<const uint4 *>(wst + r * 64 + 16 * ((2 * h + 1) ^ x));
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                const Dq8 d = make_dq8(sq[0], bq[0]);
                const uint32_t words[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    out[2 * i + 0] = dq8_pair(words[i], 0, 1, d);
                    out[2 * i + 1] = dq8_pair(words[i], 2, 3, d);
                }
            }
            tmem_st_32x32b_x16(tmem_base + t_lane + (uint32_t)(Cfg::kACol0 + s * 32 + 16 * h), out);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[s]);
#pragma unroll
            for (int i = 0; i + 1 < kSbAhead; ++i) {
                sq[i] = sq[i + 1];
                bq[i] = bq[i + 1];
            }
            load_sb(kb + 2 * kSbAhead, sq[kSbAhead - 1], bq[kSbAhead - 1]);
        }
        // ------------------------------------------------ epilogue
        const bool ok = mbar_wait_or_abort(accfull, 0, abort, prm.err) && !*abort;
        if (ok) tc_fence_after();
        const int part = warp >> 2;  // 16-token chunks part, part + 4, ...
        if constexpr (UP) {
            // Warp pair (q, q + 2) of a part: the up warp hands its 16 columns
            // to the gate warp through shared memory (the stages are idle now).
            // 16-token chunks are dealt round-robin to the four parts.  With a
            // whole 64-column block and aligned rows, h is staged as [token][64]
            // bf16 and leaves through 16-row TMA stores (a box never reaches past
            // the tile's own rows) plus 16-byte stores for the last count % 16.
            const bool is_up = q >= 2;
            const int pair_id = part * 2 + (q & 1);
            float *xbuf = reinterpret_cast<float *>(xs) + pair_id * (2 * 16 * 32);
            uint8_t *hstage = xs + kXchgBytes;
            uint16_t *hout = static_cast<uint16_t *>(prm.y);
            const bool staged = prm.h_map && nbase + kBlockW / 2 <= prm.N;
            const int nchunks = (cnt + 15) >> 4;
            int it = 0;
            for (int ch = part; ch < nchunks; ch += 4, ++it) {
                const int c0 = ch * 16;
                uint32_t acc[16];
                if (ok) {
                    tmem_ld_32x32b_x16(tmem_base + t_lane + (uint32_t)c0, acc);
                    tmem_ld_wait();
                }
                float *buf = xbuf + (it & 1) * (16 * 32);
                if (is_up && ok) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) buf[j * 32 + lane] = __uint_as_float(acc[j]);
                }
                bar_sync(1 + pair_id, 64);
                if (!is_up && ok && row_ok) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int col = c0 + j;
                        if (col < cnt) {
                            const uint16_t hv =
                                f32_to_bf16(silu_f32(__uint_as_float(acc[j])) * buf[j * 32 + lane]);
                            if (staged)
                                *reinterpret_cast<uint16_t *>(hstage + col * 128 + r * 2) = hv;
                            else
                                hout[(int64_t)(g0 + col) * prm.y_ld + nrow] = hv;
                        }
                    }
                }
            }
            if (staged) {
                fence_proxy_async_smem();
                bar_sync(9, 16 * 32);
                if (ok) {
                    const int groups = cnt >> 4;
                    if (threadIdx.x == 0) {
                        for (int gi = 0; gi < groups; ++gi)
                            tma_store_2d(&tmap_h, hstage + gi * 16 * 128, (int32_t)nbase,
                                         (int32_t)(g0 + gi * 16));
                        bulk_commit_group();
                    }
                    const int rest0 = groups * 16;
                    for (int v = threadIdx.x; v < (cnt - rest0) * 8; v += 16 * 32) {
                        const int col = rest0 + (v >> 3), ck = v & 7;
                        *reinterpret_cast<uint4 *>(hout + (int64_t)(g0 + col) * prm.y_ld + nbase +
                                                   ck * 8) =
                            *reinterpret_cast<const uint4 *>(hstage + col * 128 + ck * 16);
                    }
                    if (threadIdx.x == 0) bulk_wait_group_read0();
                }
            }
        } else {
            float *dout = static_cast<float *>(prm.y);
            if (ok) {
                const int nchunks = (cnt + 15) >> 4;
                for (int ch = part; ch < nchunks; ch += 4) {
                    const int c0 = ch * 16;
                    uint32_t acc[16];
                    tmem_ld_32x32b_x16(tmem_base + t_lane + (uint32_t)c0, acc);
                    tmem_ld_wait();
                    if (row_ok) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int col = c0 + j;
                            if (col < cnt)
                                dout[(int64_t)rows[col] * prm.y_ld + nrow] = __uint_as_float(acc[j]);
                        }
                    }
                }
            }
            if (prm.fuse) {
                // Fused score-weighted combine.  Each of this tile's pairs
                // counts itself in for its token and this n-block; the CTA
                // that brings a token's count to its number of routed pairs
                // sums the token's pairs, in slot order, exactly as the
                // separate combine did -- so the result does not depend on
                // which CTA finishes last.  No CTA waits for another.
                int *list = reinterpret_cast<int *>(xs);  // the ring is idle now
                int *nlist = list + kMaxTok;
                __threadfence();  // this thread's d stores before its arrivals
                if (threadIdx.x == 0) *nlist = 0;
                bar_sync(9, 16 * 32);
                if (ok && (int)threadIdx.x < cnt) {
                    const int p = rows[threadIdx.x];
                    const int t = p / prm.top_k;
                    int kv = 0;
                    for (int j = 0; j < prm.top_k; ++j) {
                        const int l = prm.idx[(int64_t)t * prm.top_k + j] - prm.e0;
                        kv += (l >= 0 && l < prm.ne) ? 1 : 0;
                    }
                    const int64_t ci = (int64_t)t * gridDim.x + blockIdx.x;
                    if (atomicAdd(&prm.cnt[ci], 1) == kv - 1) {
                        list[atomicAdd(nlist, 1)] = t;
                        prm.cnt[ci] = 0;  // ready for the next call
                    }
                }
                bar_sync(9, 16 * 32);
                __threadfence();
                const int L = *nlist;
                const int64_t n = nbase + lane * 4;  // 4 columns per lane, 128 per warp
                for (int i = warp; i < L; i += 16) {
                    const int t = list[i];
                    if (n >= prm.N) continue;
                    float *ro_dst = nullptr;
                    if (prm.ro.n > 0) {
                        const int64_t q = t / prm.ro.per, r = t % prm.ro.per;
                        if (r >= prm.ro.count[q]) continue;  // padding row
                        ro_dst = prm.ro.dst[q] + (prm.ro.row0 + r) * prm.N + n;
                    }
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int j = 0; j < prm.top_k; ++j) {
                        const int64_t pj = (int64_t)t * prm.top_k + j;
                        const int l = prm.idx[pj] - prm.e0;
                        if (l < 0 || l >= prm.ne) continue;
                        const float sc = bf16_to_f32(f32_to_bf16(prm.scores[pj]));
                        const float4 v = __ldcg(reinterpret_cast<const float4 *>(dout + pj * prm.y_ld + n));
                        acc.x = __fmaf_rn(sc, v.x, acc.x);
                        acc.y = __fmaf_rn(sc, v.y, acc.y);
                        acc.z = __fmaf_rn(sc, v.z, acc.z);
                        acc.w = __fmaf_rn(sc, v.w, acc.w);
                    }
                    if (ro_dst) {
                        *reinterpret_cast<float4 *>(ro_dst) = acc;
                    } else {
                        uint2 o;
                        o.x = (uint32_t)f32_to_bf16(acc.x) | ((uint32_t)f32_to_bf16(acc.y) << 16);
                        o.y = (uint32_t)f32_to_bf16(acc.z) | ((uint32_t)f32_to_bf16(acc.w) << 16);
                        *reinterpret_cast<uint2 *>(prm.out + (int64_t)t * prm.N + n) = o;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        if (*abort) {
            // let tensor-core work and copies still in flight finish before freeing TMEM
            const unsigned long long t0 = global_timer_ns();
            while (global_timer_ns() - t0 < 10000000ull) {
            }
        }
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

template <int BITS, bool UP>
cudaError_t launch_cfg(const TcMoeArgs &a, cudaStream_t stream) {
    using Cfg = MoeCfg<BITS>;
    const uint64_t Kw = (uint64_t)a.K * BITS / 32;
    const uint64_t wrows = (uint64_t)a.E * (uint64_t)a.N;
    const uint32_t wbox_rows = UP ? kBlockW / 2 : kBlockW;
    const CUtensorMapSwizzle wsw = BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUtensorMap m1, m2, mx;
    if (!make_map_2d(&m1, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w1, Kw, wrows, Kw * 4,
                     kBlockK * BITS / 32, wbox_rows, wsw))
        return cudaErrorInvalidValue;
    m2 = m1;  // unused by the down kernel
    if (UP && !make_map_2d(&m2, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w2, Kw, wrows, Kw * 4,
                           kBlockK * BITS / 32, wbox_rows, wsw))
        return cudaErrorInvalidValue;
    if (!make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, (uint64_t)a.K,
                     (uint64_t)a.x_rows_total, (uint64_t)a.x_ld * 2, kBlockK, kMaxTok,
                     CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    // up: h [P, N] bf16 through 16-row TMA stores when its rows are 16-byte aligned
    CUtensorMap mh = mx;
    const bool h_map = UP && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.y_ld % 8 == 0 &&
                       make_map_2d(&mh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.y, (uint64_t)a.N,
                                   (uint64_t)a.x_rows_total, (uint64_t)a.y_ld * 2, kBlockW / 2, 16,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!h_map) mh = mx;  // unused
    MoeTcParams prm;
    prm.h_map = h_map ? 1 : 0;
    prm.N = a.N;
    prm.K = a.K;
    prm.G = a.K / a.gs;
    prm.gs_shift = a.gs == 32 ? 5 : (a.gs == 64 ? 6 : 7);
    prm.num_kb = (int)(a.K / kBlockK);
    prm.s = a.s1;
    prm.b = a.b1;
    prm.s2 = a.s2;
    prm.b2 = a.b2;
    prm.tiles = a.tiles;
    prm.n_tiles = a.n_tiles;
    prm.rows = a.rows;
    prm.y = a.y;
    prm.y_ld = a.y_ld;
    prm.err = device_error_word();
    prm.fuse = !UP && a.fuse_cnt ? 1 : 0;
    prm.idx = a.idx;
    prm.scores = a.scores;
    prm.top_k = a.top_k;
    prm.e0 = a.e0;
    prm.ne = (int)a.E;
    prm.cnt = a.fuse_cnt;
    prm.out = a.out;
    prm.ro = a.ro;
    auto kern = tc_moe_kernel<BITS, UP>;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)((a.N + wbox_rows - 1) / wbox_rows), (unsigned)a.max_tiles, 1);
    kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(m1, m2, mx, mh, prm);
    return cudaGetLastError();
}

}  // namespace

bool tc_moe_supported(int bits, int gs, int64_t H, int64_t I, int64_t E, const void *x,
                      int64_t x_ld) {
    if (bits != 4 && bits != 8) return false;
    if (gs != 32 && gs != 64 && gs != 128) return false;
    if (H % kBlockK || I % kBlockK) return false;         // whole stages along both K
    if ((reinterpret_cast<uintptr_t>(x) & 15) || x_ld % 8) return false;  // 16-byte row copies
    if (E * (H > I ? H : I) > ((int64_t)1 << 31) - 1) return false;      // TMA row coordinate
    return tensor_maps_available();
}

cudaError_t launch_tc_moe(const TcMoeArgs &a, cudaStream_t stream) {
    if (a.max_tiles <= 0) return cudaSuccess;
    if (a.up)
        return a.bits == 4 ? launch_cfg<4, true>(a, stream) : launch_cfg<8, true>(a, stream);
    return a.bits == 4 ? launch_cfg<4, false>(a, stream) : launch_cfg<8, false>(a, stream);
}

}  // namespace nq
