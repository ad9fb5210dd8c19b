// gemm_tc.cu -- prefill quantized GEMM on the 5th-generation tensor cores.
//
//   y[m, n] = sum_k x[m, k] * w_hat[n, k]   (w_hat = MLX dequantized bf16)
//
// Tile: 128 weight rows (the UMMA M side) x BM tokens (the UMMA N side) per
// CTA, K consumed 64 codes per pipeline stage.  Roles (18 warps):
//   warp 16     TMA producer: per stage one box of activations
//               [BM rows x 64 bf16] (128-byte swizzle, the canonical K-major
//               UMMA layout) and one box of packed codes [128 rows x 32 or
//               64 bytes] (32/64-byte swizzle so that the dequant reads are
//               bank-conflict free);
//   warps 0..15 dequantizers: lane r of warp w owns weight row 32*(w%4)+r,
//               half (w/4)%2 of the stage's 64 codes, and the stages of parity
//               w/8 (two stages are dequantized at once, so the per-stage
//               latency of the smem read -> dequant -> tcgen05.st chain is
//               hidden behind the MMA of the previous stage); the codes become
//               exact MLX bf16 values in registers and go straight into tensor
//               memory with tcgen05.st -- the weights are the MMA's A operand
//               *in TMEM*, so they never round-trip through shared memory;
//   warp 17     TMEM allocator and the single MMA-issuing thread:
//               tcgen05.mma.cta_group::1.kind::f16, A from TMEM, B (tokens)
//               from shared memory, fp32 accumulator (128 lanes x BM columns)
//               in TMEM; tcgen05.commit releases stages back to the producer.
//   Epilogue: warps 0..15 read the accumulator with tcgen05.ld (lane = weight
//   row, column = token; a quarter of the columns each), stage the bf16 tile
//   in the (now idle) ring's shared memory and one thread writes it with a
//   TMA tensor store -- the CTA leaves as soon as the store has read shared
//   memory.  (Tensor-parallel fan-out and outputs a tensor map cannot
//   describe keep per-thread stores.)
// Wave tail: one CTA fits an SM, so a tile count just above a multiple of the
// SM count leaves a last wave of a few CTAs that takes as long as a full one
// (2048 x 14336 at 256 x 128 tiles: 896 = 6 x 148 + 8).  The last `rem` tiles
// are split along K over a cluster of S CTAs each (S = 2, 4 or 8).  Every CTA
// of a cluster stages its fp32 partial tile in its own shared memory (free
// once the main loop is done); after a cluster barrier each CTA sums 1/S of
// the tile's tokens over the S partials through distributed shared memory and
// stores them.  The split kernel is launched first and lets the whole-tile
// grid start beside it (programmatic dependent launch), so the tail runs on a
// few SMs while the others already work through the whole tiles.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

constexpr int kBlockW = 128;     // weight rows per CTA (UMMA M)
constexpr int kBlockK = 64;      // codes per stage
constexpr int kSbAhead = 2;       // scale/bias prefetch depth, in this warp's iterations
constexpr int kStageArrivals = 8;   // of the 16 dequant warps, those working on one stage
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;
constexpr int kThreads = 576;
constexpr int kSplitMax = 8;      // CTAs (one cluster) per split tail tile, at most

template <int BITS, int BM>
struct TcCfg {
    static constexpr int kXStageBytes = BM * kBlockK * 2;             // bf16 tokens
    static constexpr int kWStageBytes = kBlockW * kBlockK * BITS / 8;  // packed codes
    static constexpr int kStageBytes = kXStageBytes + kWStageBytes;
    static constexpr int kStages = (BM == 256) ? (BITS == 4 ? 6 : 5) : (BM == 128 ? 8 : 10);
    static constexpr int kACol0 = BM;                                  // first A-stage column
    static constexpr int kTmemCols = 512;
    static_assert(kACol0 + kStages * 32 <= kTmemCols, "TMEM budget");
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 512 /*barriers*/;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct TcParams {
    int64_t M, N, K, x_ld, y_ld;
    int gs_shift;  // log2(group size)
    int num_kb;
    int n_tiles;      // weight-row tiles; tile t: rows (t % n_tiles) * 128, tokens (t / n_tiles) * BM
    int main_tiles;   // tiles computed whole, one CTA each; the rest are split along K
    int split;        // CTAs (one cluster) per split tile: 2, 4 or 8
    int tma_store;    // whole tiles leave through the y tensor map
    int push_vec;     // fan-out of whole tiles by 16-byte stores (rows of y 16-byte aligned)
    const uint16_t *s, *b;
    uint16_t *y;
    unsigned int *err;
    PushDev push;  // tensor-parallel fan-out of the stores (n == 0: local only)
};

// Every thread of every CTA of the cluster.  The non-.aligned form: the
// producer and MMA warps arrive right after loops that only one lane ran.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// 16 bytes of CTA `rank`'s shared memory at the offset of `local` in this CTA
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote)
                 : "memory");
    return v;
}

__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort,
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

// SPLIT = false: one CTA per tile on the (weight tile, token tile) grid.
// SPLIT = true: the tail -- a 1-D grid of prm.split CTAs per tile, for the
// tiles from prm.main_tiles on.
template <int BITS, int BM, bool SPLIT, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    tc_qgemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_y, const TcParams prm) {
    using Cfg = TcCfg<BITS, BM>;
    constexpr int S = Cfg::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint8_t *xs = smem;                               // S x [BM][128 B]
    uint8_t *ws = smem + S * Cfg::kXStageBytes;       // S x [128][32|64 B]
    uint64_t *bars = reinterpret_cast<uint64_t *>(ws + S * Cfg::kWStageBytes);
    uint64_t *full = bars;            // TMA landed (x + w)
    uint64_t *empty = bars + S;       // stage free: MMA done (1) + dequant read (8 warps)
    uint64_t *afull = bars + 2 * S;   // A written to TMEM (8 warps)
    uint64_t *accfull = bars + 3 * S; // accumulator complete
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 3 * S + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // tile origin and this CTA's k-blocks [kb0, kb0 + num_kb).  (The whole-tile
    // instance reads the origin straight from blockIdx: deriving it by division
    // measurably slows the main loop.)
    int tile = 0, ks = 0, nsplit = 1, kb0 = 0, num_kb = prm.num_kb;
    int64_t n0 = (int64_t)blockIdx.x * kBlockW, m0 = (int64_t)blockIdx.y * BM;
    if constexpr (!SPLIT) {
        // the last row's tail tiles belong to the split launch (uniform over the CTA,
        // before any barrier or TMEM)
        if ((int)(blockIdx.y * gridDim.x + blockIdx.x) >= prm.main_tiles) return;
    } else {
        // the whole-tile grid is launched after this one as a programmatic
        // dependent: let it fill the other SMs now
        pdl_launch_dependents();
        nsplit = prm.split;
        tile = prm.main_tiles + (int)blockIdx.x / nsplit;
        ks = (int)blockIdx.x % nsplit;
        n0 = (int64_t)(tile % prm.n_tiles) * kBlockW;
        m0 = (int64_t)(tile / prm.n_tiles) * BM;
        kb0 = (int)(((int64_t)ks * prm.num_kb) / nsplit);
        num_kb = (int)(((int64_t)(ks + 1) * prm.num_kb) / nsplit) - kb0;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kStageArrivals);
            mbar_init(&afull[s], kStageArrivals);
        }
        mbar_init(accfull, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == kProducerWarp && lane == 0) {
        prefetch_tmap(&tmap_x);
        prefetch_tmap(&tmap_w);
        if (!SPLIT && prm.tma_store) prefetch_tmap(&tmap_y);
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
            const uint32_t bytes = Cfg::kXStageBytes + Cfg::kWStageBytes;
            for (int i = 0; i < num_kb; ++i) {
                const int s = i % S;
                const uint32_t ph = (uint32_t)(i / S) & 1u;
                const int kb = kb0 + i;
                if (!wait_or_abort(&empty[s], ph ^ 1u, abort, prm.err)) break;
                mbar_expect_tx(&full[s], bytes);
                tma_load_2d(xs + s * Cfg::kXStageBytes, &tmap_x, &full[s], kb * kBlockK, (int32_t)m0);
                tma_load_2d(ws + s * Cfg::kWStageBytes, &tmap_w, &full[s],
                            kb * (kBlockK * BITS / 32), (int32_t)n0);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            constexpr uint32_t idesc = F16 ? idesc_f16_f32(kBlockW, BM) : idesc_bf16_f32(kBlockW, BM);
            for (int i = 0; i < num_kb; ++i) {
                const int s = i % S;
                const uint32_t ph = (uint32_t)(i / S) & 1u;
                if (!wait_or_abort(&full[s], ph, abort, prm.err)) break;
                if (!wait_or_abort(&afull[s], ph, abort, prm.err)) break;
                tc_fence_after();
                const uint64_t bdesc = smem_desc_k_sw128(smem_u32(xs + s * Cfg::kXStageBytes));
#pragma unroll
                for (int j = 0; j < kBlockK / 16; ++j) {
                    const uint32_t a_tmem = tmem_base + (uint32_t)(Cfg::kACol0 + s * 32 + j * 8);
                    // +32 bytes per 16 bf16 of K inside the 128-byte swizzled row
                    umma_ts(tmem_base, a_tmem, bdesc + (uint64_t)(j * 2), idesc,
                            (i > 0 || j > 0) ? 1u : 0u);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(accfull);
        }
    } else {
        // ------------------------------------------------ dequantizers
        const int q = warp & 3;          // TMEM lane quadrant
        const int h = (warp >> 2) & 1;   // which 32 codes of the stage
        const int par = warp >> 3;       // which stages: (kb - kb0) % 2 == par
        const int r = q * 32 + lane;     // weight row inside the tile
        const int64_t n = n0 + r;
        const bool row_ok = n < prm.N;
        const int64_t G = prm.K >> prm.gs_shift;
        const uint16_t *srow = prm.s + (row_ok ? n : 0) * G;
        const uint16_t *brow = prm.b + (row_ok ? n : 0) * G;
        auto load_sb = [&](int kb, uint16_t &sv, uint16_t &bv) {
            const int k = kb * kBlockK + 32 * h;
            sv = 0;
            bv = 0;
            if (row_ok && kb < kb0 + num_kb && k < prm.K) {
                sv = srow[k >> prm.gs_shift];
                bv = brow[k >> prm.gs_shift];
            }
        };
        // Scale and bias of this thread's row for its next kSbAhead stages, in
        // a shift register: the load for a stage is issued kSbAhead of this
        // warp's iterations before its use, which covers an HBM round trip.
        uint16_t sq[kSbAhead], bq[kSbAhead];
#pragma unroll
        for (int i = 0; i < kSbAhead; ++i) load_sb(kb0 + par + 2 * i, sq[i], bq[i]);
        const uint32_t t_lane = (uint32_t)(q * 32) << 16;
        for (int it = par; it < num_kb; it += 2) {
            const int kb = kb0 + it;
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            if (!wait_or_abort(&full[s], ph, abort, prm.err)) break;
            tc_fence_after();
            uint32_t out[16];
            const uint8_t *wst = ws + s * Cfg::kWStageBytes;
            if constexpr (BITS == 4) {
                // row r: 32 bytes; chunk h, 32-byte swizzle: chunk ^= (r >> 2) & 1
                const uint4 v = *reinterpret_cast<const uint4 *>(
                    wst + r * 32 + 16 * (h ^ ((r >> 2) & 1)));
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                const Dq4 d = F16 ? Dq4{} : make_dq4(sq[0], bq[0]);
                const Dq4h dh = make_dq4h(sq[0], bq[0]);
                const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint32_t d0, d1, d2, d3;
                    if constexpr (F16) {
                        d0 = dqh_pair(q4_pair_biased_h(words[i], 0), dh);
                        d1 = dqh_pair(q4_pair_biased_h(words[i], 1), dh);
                        d2 = dqh_pair(q4_pair_biased_h(words[i], 2), dh);
                        d3 = dqh_pair(q4_pair_biased_h(words[i], 3), dh);
                    } else {
                        d0 = dq4_pair(q4_pair_biased(words[i], 0), d);  // (w0, w4)
                        d1 = dq4_pair(q4_pair_biased(words[i], 1), d);  // (w1, w5)
                        d2 = dq4_pair(q4_pair_biased(words[i], 2), d);  // (w2, w6)
                        d3 = dq4_pair(q4_pair_biased(words[i], 3), d);  // (w3, w7)
                    }
                    out[4 * i + 0] = prmt(d0, d1, 0x5410u);  // (w0, w1)
                    out[4 * i + 1] = prmt(d2, d3, 0x5410u);  // (w2, w3)
                    out[4 * i + 2] = prmt(d0, d1, 0x7632u);  // (w4, w5)
                    out[4 * i + 3] = prmt(d2, d3, 0x7632u);  // (w6, w7)
                }
            } else {
                // row r: 64 bytes; chunks 2h, 2h+1, 64-byte swizzle: chunk ^= (r >> 1) & 3
                const int x = (r >> 1) & 3;
                const uint4 v0 = *reinterpret_cast<const uint4 *>(wst + r * 64 + 16 * ((2 * h) ^ x));
                const uint4 v1 =
                    *reinterpret_cast<const uint4 *>(wst + r * 64 + 16 * ((2 * h + 1) ^ x));
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                const uint32_t words[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                if constexpr (F16) {
                    const Dq4h dh = make_dq4h(sq[0], bq[0]);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        out[2 * i + 0] = dqh_pair(q8_pair_biased_h(words[i], 0, 1), dh);
                        out[2 * i + 1] = dqh_pair(q8_pair_biased_h(words[i], 2, 3), dh);
                    }
                } else {
                    const Dq8 d = make_dq8(sq[0], bq[0]);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        out[2 * i + 0] = dq8_pair(words[i], 0, 1, d);
                        out[2 * i + 1] = dq8_pair(words[i], 2, 3, d);
                    }
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
        bool acc_ok = wait_or_abort(accfull, 0, abort, prm.err) && !*abort;
        const int part = warp >> 2;  // quarter of the accumulator columns
        if constexpr (SPLIT) {
            // the partial tile into this CTA's shared memory, [token][row] fp32
            // (every MMA and every dequantizer read of the ring is done)
            float *part_sm = reinterpret_cast<float *>(smem);
            if (acc_ok) {
                tc_fence_after();
                for (int c0 = part * (BM / 4); c0 < (part + 1) * (BM / 4); c0 += 16) {
                    uint32_t acc[16];
                    tmem_ld_32x32b_x16(tmem_base + t_lane + (uint32_t)c0, acc);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) part_sm[(c0 + j) * kBlockW + r] = __uint_as_float(acc[j]);
                }
            }
            acc_ok = false;
        }
        if (!SPLIT && prm.tma_store) {
            // bf16 tile [BM tokens][128 rows] in shared memory, then one TMA store
            uint8_t *stage = smem;
            if (acc_ok) {
                tc_fence_after();
                for (int c0 = part * (BM / 4); c0 < (part + 1) * (BM / 4); c0 += 16) {
                    uint32_t acc[16];
                    tmem_ld_32x32b_x16(tmem_base + t_lane + (uint32_t)c0, acc);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        *reinterpret_cast<uint16_t *>(stage + ((c0 + j) * kBlockW + r) * 2) =
                            f32_to_t16<F16>(__uint_as_float(acc[j]));
                }
            }
            fence_proxy_async_smem();
            bar_sync(1, 16 * 32);
            if (threadIdx.x == 0 && acc_ok) {
                tma_store_2d(&tmap_y, stage, (int32_t)n0, (int32_t)m0);
                bulk_commit_group();
                bulk_wait_group_read0();
            }
            acc_ok = false;
        }
        if (!SPLIT && prm.push.n && prm.push_vec) {
            // Tensor-parallel fan-out: the bf16 tile [BM tokens][128 rows] is
            // staged in the idle ring, then every thread pushes 16-byte pieces of
            // token rows (256 contiguous bytes of y each) to every rank's y.
            uint8_t *stage = smem;
            if (acc_ok) {
                tc_fence_after();
                for (int c0 = part * (BM / 4); c0 < (part + 1) * (BM / 4); c0 += 16) {
                    uint32_t acc[16];
                    tmem_ld_32x32b_x16(tmem_base + t_lane + (uint32_t)c0, acc);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        *reinterpret_cast<uint16_t *>(stage + ((c0 + j) * kBlockW + r) * 2) =
                            f32_to_t16<F16>(__uint_as_float(acc[j]));
                }
            }
            bar_sync(1, 16 * 32);
            // every lane of every storing warp takes part in the (bounded) wait
            const bool ready = push_wait_ready(prm.push, prm.err);
            if (acc_ok && ready) {
                const int64_t rows_left = prm.N - n0;
                for (int q = threadIdx.x; q < BM * (kBlockW / 8); q += 16 * 32) {
                    const int tok = q / (kBlockW / 8), ch = q % (kBlockW / 8);
                    const int64_t m = m0 + tok;
                    if (m >= prm.M || ch * 8 >= rows_left) continue;
                    const uint4 v = *reinterpret_cast<const uint4 *>(stage + (tok * kBlockW + ch * 8) * 2);
                    uint16_t *dst = prm.y + m * prm.y_ld + n0 + ch * 8;
                    if (ch * 8 + 8 <= rows_left) {
                        push_store(prm.push, reinterpret_cast<uint4 *>(dst), v);
                    } else {
                        const uint16_t *e = reinterpret_cast<const uint16_t *>(&v);
                        for (int i = 0; i < rows_left - ch * 8; ++i) push_store(prm.push, dst + i, e[i]);
                    }
                }
            }
            acc_ok = false;
        }
        if (prm.push.n && acc_ok && !push_wait_ready(prm.push, prm.err)) acc_ok = false;
        if (acc_ok) {
            tc_fence_after();
            const int64_t nrow = n0 + r;
            for (int c0 = part * (BM / 4); c0 < (part + 1) * (BM / 4); c0 += 16) {
                uint32_t acc[16];
                tmem_ld_32x32b_x16(tmem_base + t_lane + (uint32_t)c0, acc);
                tmem_ld_wait();
                if (nrow < prm.N) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int64_t m = m0 + c0 + j;
                        if (m < prm.M)
                            push_store(prm.push, prm.y + m * prm.y_ld + nrow,
                                       f32_to_t16<F16>(__uint_as_float(acc[j])));
                    }
                }
            }
        }
    }

    if constexpr (SPLIT) {
        // sum this CTA's share of the tile's tokens over the cluster's partials
        cluster_sync_all();
        const int tpc = BM / nsplit;
        const int tok0 = ks * tpc;
        bool store_ok = !*abort;
        if (prm.push.n && !push_wait_ready(prm.push, prm.err)) store_ok = false;
        const uint32_t part_u32 = smem_u32(smem);
        for (int qd = threadIdx.x; qd < tpc * (kBlockW / 4); qd += kThreads) {
            const int tok = tok0 + qd / (kBlockW / 4);
            const int row = (qd % (kBlockW / 4)) * 4;
            const uint32_t off = part_u32 + (uint32_t)((tok * kBlockW + row) * 4);
            float4 src[kSplitMax];
#pragma unroll
            for (int c = 0; c < kSplitMax; ++c)
                src[c] = c < nsplit ? ld_dsmem_f4(off, (uint32_t)c) : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 v = src[0];
#pragma unroll
            for (int c = 1; c < kSplitMax; ++c) {
                v.x += src[c].x;
                v.y += src[c].y;
                v.z += src[c].z;
                v.w += src[c].w;
            }
            const int64_t m = m0 + tok, nr = n0 + row;
            if (!store_ok || m >= prm.M) continue;
            uint16_t *dst = prm.y + m * prm.y_ld + nr;
            if (nr + 4 <= prm.N && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
                const uint2 pk = make_uint2(pack_t2<F16>(v.x, v.y), pack_t2<F16>(v.z, v.w));
                push_store(prm.push, reinterpret_cast<uint2 *>(dst), pk);
            } else {
                const float e[4] = {v.x, v.y, v.z, v.w};
                for (int i = 0; i < 4; ++i)
                    if (nr + i < prm.N) push_store(prm.push, dst + i, f32_to_t16<F16>(e[i]));
            }
        }
        cluster_sync_all();  // the peers' reads of this CTA's partial are done
    } else {
        // (launched after the split tail as its programmatic dependent: completing
        // only after the tail grid keeps the stream's order for later work)
        if (prm.split > 1) pdl_wait();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        if (*abort) {
            // let any tensor-core work still in flight finish before freeing TMEM
            const unsigned long long t0 = global_timer_ns();
            while (global_timer_ns() - t0 < 10000000ull) {
            }
        }
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ----------------------------------------------------------------------------
// CTA-pair kernel for the whole tiles of problems with 256-token tiles: two
// CTAs (a cluster on two SMs) own 256 weight rows (128 each) x 256 tokens.
// One tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16) reads both operands
// from shared memory -- each CTA holds its 128 weight rows of A and its 128
// tokens of B -- and writes each CTA's 128 x 256 fp32 accumulator in its own
// TMEM.  Compared with the single-CTA kernel above, the dequantized weights go
// to shared memory (16-byte st.shared into the canonical K-major layout, 128-
// byte swizzle) instead of TMEM, and every SM reads only half of the token
// tile per MMA, so the shared-memory traffic per MMA stays at the single-CTA
// kernel's while the A-operand stores into TMEM are gone.
//   warp 16  TMA producer (each CTA): its token half [128 x 64 bf16] and its
//            code tile [128 rows x 32|64 B] per stage;
//   warps 0..15 dequantizers (each CTA), as in the single-CTA kernel, writing
//            A into the stage's A slot; the 8 warps of a stage then arrive on
//            their own CTA's afull barrier;
//   warp 17  allocates 256 TMEM columns over the pair (cta_group::2).  In the
//            odd CTA one lane forwards each completed afull phase to the even
//            CTA's peer barrier (one remote arrival per stage, from a thread
//            with no loads in flight: a cluster-scope release waits for the
//            releasing thread's outstanding loads, and the dequantizers always
//            have scale prefetches in flight).  In the even CTA one lane waits
//            for both, issues the MMAs and commits each stage to the empty
//            barriers of both CTAs (multicast commit).
// The epilogue is the single-CTA kernel's TMA-store epilogue, per CTA.
// ----------------------------------------------------------------------------
constexpr int kPairTok = 256;   // tokens per pair tile (UMMA N)
constexpr int kPairHalf = 128;  // tokens staged by each CTA

template <int BITS>
struct PairCfg {
    static constexpr int kXBytes = kPairHalf * kBlockK * 2;             // 16 KB
    static constexpr int kABytes = kBlockW * kBlockK * 2;               // 16 KB
    static constexpr int kWBytes = kBlockW * kBlockK * BITS / 8;        // 4 | 8 KB
    static constexpr int kStages = 5;
    static constexpr int kSmemBytes =
        kStages * (kXBytes + kABytes + kWBytes) + 1024 /*align*/ + 512 /*barriers*/;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    static_assert(kPairTok * kBlockW * 2 <= kStages * (kXBytes + kABytes), "epilogue staging");
};

template <int BITS>
__global__ void __launch_bounds__(kThreads, 1)
    tc_qgemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_x,
                         const __grid_constant__ CUtensorMap tmap_w,
                         const __grid_constant__ CUtensorMap tmap_y, const TcParams prm) {
    using Cfg = PairCfg<BITS>;
    constexpr int S = Cfg::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint8_t *as = smem;                                   // S x A slot [128 rows][128 B], SW128
    uint8_t *xs = smem + S * Cfg::kABytes;                // S x [128 tokens][128 B], SW128
    uint8_t *ws = xs + S * Cfg::kXBytes;                  // S x [128 rows][32|64 B]
    uint64_t *bars = reinterpret_cast<uint64_t *>(ws + S * Cfg::kWBytes);
    uint64_t *full = bars;            // this CTA's TMA landed (x half + codes)
    uint64_t *empty = bars + S;       // the pair's MMAs of the stage completed
    uint64_t *afull = bars + 2 * S;   // this CTA's A slot written (8 warps)
    uint64_t *accfull = bars + 3 * S; // accumulator complete
    uint64_t *pafull = bars + 3 * S + 1;  // (even CTA) the odd CTA's A slot written
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 4 * S + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // both CTAs of a pair see the same tile index (even n-tile, same row)
    if ((int)(blockIdx.y * gridDim.x + (blockIdx.x & ~1u)) >= prm.main_tiles) return;
    const uint32_t rank = cluster_ctarank();
    const int64_t n0 = (int64_t)blockIdx.x * kBlockW;  // this CTA's 128 weight rows
    const int64_t m0 = (int64_t)blockIdx.y * kPairTok;  // the pair's 256 tokens
    const int num_kb = prm.num_kb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&afull[s], kStageArrivals);
            mbar_init(&pafull[s], 1);
        }
        mbar_init(accfull, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == kProducerWarp && lane == 0) {
        prefetch_tmap(&tmap_x);
        prefetch_tmap(&tmap_w);
        prefetch_tmap(&tmap_y);
    }
    if (warp == kMmaWarp) {
        tmem_alloc_pair(tmem_holder, kPairTok);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            const uint32_t bytes = Cfg::kXBytes + Cfg::kWBytes;
            for (int i = 0; i < num_kb; ++i) {
                const int s = i % S;
                const uint32_t ph = (uint32_t)(i / S) & 1u;
                if (!wait_or_abort(&empty[s], ph ^ 1u, abort, prm.err)) break;
                mbar_expect_tx(&full[s], bytes);
                tma_load_2d(xs + s * Cfg::kXBytes, &tmap_x, &full[s], i * kBlockK,
                            (int32_t)(m0 + kPairHalf * rank));
                tma_load_2d(ws + s * Cfg::kWBytes, &tmap_w, &full[s], i * (kBlockK * BITS / 32),
                            (int32_t)n0);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0 && rank == 1) {
            // forward each afull phase of this CTA to the even CTA
            const uint32_t peer0 = mapa_shared(smem_u32(pafull), 0);
            for (int i = 0; i < num_kb; ++i) {
                const int s = i % S;
                if (!wait_or_abort(&afull[s], (uint32_t)(i / S) & 1u, abort, prm.err)) break;
                mbar_arrive_cluster(peer0 + (uint32_t)(s * 8));
            }
        }
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(2 * kBlockW, kPairTok);
            for (int i = 0; i < num_kb; ++i) {
                const int s = i % S;
                const uint32_t ph = (uint32_t)(i / S) & 1u;
                if (!wait_or_abort(&afull[s], ph, abort, prm.err)) break;
                bool ok = mbar_try_wait_cluster(&pafull[s], ph);
                if (!ok) {
                    const unsigned long long t0 = global_timer_ns();
                    while (!(ok = mbar_try_wait_cluster(&pafull[s], ph))) {
                        if (*abort) break;
                        if (global_timer_ns() - t0 > kWaitLimitNs) {
                            *abort = 1;
                            atomicOr(prm.err, kErrWaitTimeout);
                            break;
                        }
                    }
                }
                if (!ok) break;
                tc_fence_after();
                const uint64_t adesc = smem_desc_k_sw128(smem_u32(as + s * Cfg::kABytes));
                const uint64_t bdesc = smem_desc_k_sw128(smem_u32(xs + s * Cfg::kXBytes));
#pragma unroll
                for (int j = 0; j < kBlockK / 16; ++j)
                    // +32 bytes per 16 bf16 of K inside the 128-byte swizzled rows
                    umma_ss_pair(tmem_base, adesc + (uint64_t)(j * 2), bdesc + (uint64_t)(j * 2),
                                 idesc, (i > 0 || j > 0) ? 1u : 0u);
                umma_commit_pair(&empty[s], 3);
            }
            umma_commit_pair(accfull, 3);
        }
    } else {
        // ------------------------------------------------ dequantizers
        const int q = warp & 3;
        const int h = (warp >> 2) & 1;
        const int par = warp >> 3;
        const int r = q * 32 + lane;     // weight row inside this CTA's 128
        const int64_t n = n0 + r;
        const bool row_ok = n < prm.N;
        const int64_t G = prm.K >> prm.gs_shift;
        const uint16_t *srow = prm.s + (row_ok ? n : 0) * G;
        const uint16_t *brow = prm.b + (row_ok ? n : 0) * G;
        auto load_sb = [&](int kb, uint16_t &sv, uint16_t &bv) {
            const int k = kb * kBlockK + 32 * h;
            sv = 0;
            bv = 0;
            if (row_ok && kb < num_kb && k < prm.K) {
                sv = srow[k >> prm.gs_shift];
                bv = brow[k >> prm.gs_shift];
            }
        };
        uint16_t sq[kSbAhead], bq[kSbAhead];
#pragma unroll
        for (int i = 0; i < kSbAhead; ++i) load_sb(par + 2 * i, sq[i], bq[i]);
        // this thread's row in the A slot: 128 B, 16-byte chunk c at (c ^ (r & 7))
        const uint32_t a_row = (uint32_t)r * 128;
        for (int it = par; it < num_kb; it += 2) {
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            if (!wait_or_abort(&full[s], ph, abort, prm.err)) break;
            uint32_t out[16];
            const uint8_t *wst = ws + s * Cfg::kWBytes;
            if constexpr (BITS == 4) {
                const uint4 v = *reinterpret_cast<const uint4 *>(
                    wst + r * 32 + 16 * (h ^ ((r >> 2) & 1)));
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
                const Dq8 d = make_dq8(sq[0], bq[0]);
                const uint32_t words[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    out[2 * i + 0] = dq8_pair(words[i], 0, 1, d);
                    out[2 * i + 1] = dq8_pair(words[i], 2, 3, d);
                }
            }
            // 32 codes = 4 chunks (4h .. 4h+3) of this row of the A slot
            uint8_t *arow = as + s * Cfg::kABytes + a_row;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                *reinterpret_cast<uint4 *>(arow + (((4 * h + j) ^ (r & 7)) << 4)) =
                    make_uint4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
            fence_proxy_async_smem();  // the pair's tensor core reads the slot
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[s]);
#pragma unroll
            for (int i = 0; i + 1 < kSbAhead; ++i) {
                sq[i] = sq[i + 1];
                bq[i] = bq[i + 1];
            }
            load_sb(it + 2 * kSbAhead, sq[kSbAhead - 1], bq[kSbAhead - 1]);
        }
        // ------------------------------------------------ epilogue
        bool acc_ok = wait_or_abort(accfull, 0, abort, prm.err) && !*abort;
        const int part = warp >> 2;  // quarter of the accumulator columns (tokens)
        const uint32_t t_lane = (uint32_t)(q * 32) << 16;
        uint8_t *stage = smem;
        if (acc_ok) {
            tc_fence_after();
            for (int c0 = part * (kPairTok / 4); c0 < (part + 1) * (kPairTok / 4); c0 += 16) {
                uint32_t acc[16];
                tmem_ld_32x32b_x16(tmem_base + t_lane + (uint32_t)c0, acc);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    *reinterpret_cast<uint16_t *>(stage + ((c0 + j) * kBlockW + r) * 2) =
                        f32_to_bf16(__uint_as_float(acc[j]));
            }
        }
        fence_proxy_async_smem();
        bar_sync(1, 16 * 32);
        if (threadIdx.x == 0 && acc_ok) {
            tma_store_2d(&tmap_y, stage, (int32_t)n0, (int32_t)m0);
            bulk_commit_group();
            bulk_wait_group_read0();
        }
    }

    // Lanes 1..31 of the producer and MMA warps wait here for their lane 0:
    // parked in the cluster barrier instead, they starve lane 0's loop (its
    // waits were observed microseconds late).
    __syncwarp();
    // (launched after the split tail as its programmatic dependent: completing
    // only after the tail grid keeps the stream's order for later work)
    if (prm.split > 1) pdl_wait();
    tc_fence_before();
    cluster_sync_all();  // both CTAs are done with their TMEM and the shared operands
    if (warp == kMmaWarp) {
        if (*abort) {
            const unsigned long long t0 = global_timer_ns();
            while (global_timer_ns() - t0 < 10000000ull) {
            }
        }
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kPairTok);
    }
}

// ------------------------------------------------------------- host side

// The CTA-pair kernel serves the whole 256-token tiles when the environment
// sets NQ_TC_PAIR=1 (both kernels compute the same tiles; the single-CTA
// kernel is the default while it is the faster one).
bool pair_kernel_enabled() {
    static const bool on = [] {
        const char *v = getenv("NQ_TC_PAIR");
        return v && v[0] == '1';
    }();
    return on;
}

// CTAs per tail tile (1: no split): the last T % W tiles (one CTA per SM on W
// SMs) are split along K when they would leave more than half the SMs idle;
// S is a power of two (it divides the token tile), at most 8 (a portable
// cluster) and leaves at least two k-blocks per CTA.
int tail_split(int64_t T, int W, int num_kb) {
    const int64_t rem = T % W;
    if (rem == 0 || rem > W / 2) return 1;
    int S = 1;
    while (S * 2 <= kSplitMax && rem * S * 2 <= W && num_kb >= 4 * S) S *= 2;
    return S;
}

// Clusters of S split-tail CTAs that can be resident at once on this device
// (asked once per device and S).
template <int BITS, int BM>
int max_clusters(int S) {
    using Cfg = TcCfg<BITS, BM>;
    constexpr int kDev = 64;
    static std::mutex mu;
    static int cache[kDev][kSplitMax + 1];
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kDev || S > kSplitMax) {
        cudaGetLastError();
        return 0;
    }
    std::lock_guard<std::mutex> lk(mu);
    if (cache[d][S] == 0) {
        auto kern = tc_qgemm_kernel<BITS, BM, true, false>;
        int clusters = 0;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Cfg::kSmemBytes) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)(S * 64), 1, 1);
            cfg.blockDim = dim3(kThreads, 1, 1);
            cfg.dynamicSmemBytes = Cfg::kSmemBytes;
            cudaLaunchAttribute attr;
            attr.id = cudaLaunchAttributeClusterDimension;
            attr.val.clusterDim.x = (unsigned)S;
            attr.val.clusterDim.y = 1;
            attr.val.clusterDim.z = 1;
            cfg.attrs = &attr;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) clusters = 0;
        }
        cudaGetLastError();
        cache[d][S] = clusters > 0 ? clusters : -1;
    }
    return cache[d][S];
}

// How a problem is cut: tiles [0, main_tiles) whole, the rest split over
// `split` CTAs each (split == 1: no split tail).
template <int BITS, int BM>
void plan_bm(const TcGemmArgs &a, int64_t *main_tiles, int *split) {
    const int64_t tiles = ((a.N + kBlockW - 1) / kBlockW) * ((a.M + BM - 1) / BM);
    const int num_kb = (int)((a.K + kBlockK - 1) / kBlockK);
    *main_tiles = tiles;
    *split = 1;
    int S = tail_split(tiles, sm_count(), num_kb);
    const int64_t rem = tiles % sm_count();
    // every cluster of the tail should be resident at once
    while (S > 1 && max_clusters<BITS, BM>(S) < rem) S /= 2;
    if (S > 1) {
        *main_tiles = tiles - rem;
        *split = S;
    }
}

template <int BITS, int BM, bool F16>
cudaError_t launch_bm(const TcGemmArgs &a, cudaStream_t stream) {
    using Cfg = TcCfg<BITS, BM>;
    constexpr CUtensorMapDataType kT16 =
        F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap mx, mw;
    const uint64_t Kw = (uint64_t)a.K * BITS / 32;
    if (!make_map_2d(&mx, kT16, a.x, (uint64_t)a.K, (uint64_t)a.M,
                     (uint64_t)a.x_ld * 2, kBlockK, BM, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    if (!make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w, Kw, (uint64_t)a.N, Kw * 4,
                     kBlockK * BITS / 32, kBlockW,
                     BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
        return cudaErrorInvalidValue;
    CUtensorMap my;
    const bool y_map = !a.push && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.y_ld % 8 == 0 &&
                       make_map_2d(&my, kT16, a.y, (uint64_t)a.N,
                                   (uint64_t)a.M, (uint64_t)a.y_ld * 2, kBlockW, BM,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!y_map) my = mx;  // unused
    TcParams prm;
    prm.tma_store = y_map ? 1 : 0;
    prm.push_vec = a.push && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.y_ld % 8 == 0 ? 1 : 0;
    prm.M = a.M;
    prm.N = a.N;
    prm.K = a.K;
    prm.x_ld = a.x_ld;
    prm.y_ld = a.y_ld;
    prm.gs_shift = a.gs == 32 ? 5 : (a.gs == 64 ? 6 : 7);
    prm.num_kb = (int)((a.K + kBlockK - 1) / kBlockK);
    prm.s = a.s;
    prm.b = a.b;
    prm.y = a.y;
    prm.err = device_error_word();
    if (a.push) prm.push = *a.push;
    const int64_t n_tiles = (a.N + kBlockW - 1) / kBlockW;
    const int64_t tiles = n_tiles * ((a.M + BM - 1) / BM);
    if (tiles > ((int64_t)1 << 30)) return cudaErrorInvalidValue;
    prm.n_tiles = (int)n_tiles;
    int64_t main_tiles = tiles;
    plan_bm<BITS, BM>(a, &main_tiles, &prm.split);
    prm.main_tiles = (int)main_tiles;
    // The split tail first (an ordinary launch: it starts after the previous
    // work on the stream), then the whole tiles on the (weight tile, token tile)
    // grid as its programmatic dependent, so that they run beside the tail.
    if (prm.split > 1) {
        cudaError_t e = cudaFuncSetAttribute(tc_qgemm_kernel<BITS, BM, true, F16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Cfg::kSmemBytes);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)((tiles - prm.main_tiles) * prm.split), 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = Cfg::kSmemBytes;
        cfg.stream = stream;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = (unsigned)prm.split;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, tc_qgemm_kernel<BITS, BM, true, F16>, mx, mw, my, prm);
        if (e != cudaSuccess) return e;
    }
    // Whole 256-token tiles go to the CTA-pair kernel when the tiles pair up
    // (an even number of 128-row weight tiles per token tile, an even count of
    // whole tiles) and the output leaves through the TMA-store epilogue.
    if constexpr (BM == kPairTok && !F16) {
        if (prm.main_tiles > 0 && pair_kernel_enabled() && n_tiles % 2 == 0 &&
            prm.main_tiles % 2 == 0 && prm.tma_store) {
            using PC = PairCfg<BITS>;
            CUtensorMap mxh;
            if (!make_map_2d(&mxh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, (uint64_t)a.K,
                             (uint64_t)a.M, (uint64_t)a.x_ld * 2, kBlockK, kPairHalf,
                             CU_TENSOR_MAP_SWIZZLE_128B))
                return cudaErrorInvalidValue;
            auto kern = tc_qgemm_pair_kernel<BITS>;
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 PC::kSmemBytes);
            if (e != cudaSuccess) return e;
            const int64_t full_rows = (prm.main_tiles + n_tiles - 1) / n_tiles;
            if (full_rows > 65535) return cudaErrorInvalidValue;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)n_tiles, (unsigned)full_rows, 1);
            cfg.blockDim = dim3(kThreads, 1, 1);
            cfg.dynamicSmemBytes = PC::kSmemBytes;
            cfg.stream = stream;
            cudaLaunchAttribute attrs[2];
            attrs[0].id = cudaLaunchAttributeClusterDimension;
            attrs[0].val.clusterDim.x = 2;
            attrs[0].val.clusterDim.y = 1;
            attrs[0].val.clusterDim.z = 1;
            attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attrs[1].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attrs;
            cfg.numAttrs = prm.split > 1 ? 2 : 1;
            e = cudaLaunchKernelEx(&cfg, kern, mxh, mw, my, prm);
            if (e != cudaSuccess) return e;
            return cudaGetLastError();
        }
    }
    if (prm.main_tiles > 0) {
        auto kern = tc_qgemm_kernel<BITS, BM, false, F16>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Cfg::kSmemBytes);
        if (e != cudaSuccess) return e;
        const int64_t full_rows = (prm.main_tiles + n_tiles - 1) / n_tiles;
        if (full_rows > 65535) return cudaErrorInvalidValue;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)n_tiles, (unsigned)full_rows, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = Cfg::kSmemBytes;
        cfg.stream = stream;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr.val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = prm.split > 1 ? 1 : 0;
        e = cudaLaunchKernelEx(&cfg, kern, mx, mw, my, prm);
        if (e != cudaSuccess) return e;
    }
    return cudaGetLastError();
}

}  // namespace

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

bool make_map_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


bool tensor_maps_available() { return encode_fn() != nullptr; }

bool tc_gemm_supported(const TcGemmArgs &a) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return false;
    if (a.bits != 4 && a.bits != 8) return false;
    // TMA: 16-byte aligned bases and row strides
    if ((reinterpret_cast<uintptr_t>(a.x) & 15) || (reinterpret_cast<uintptr_t>(a.w) & 15))
        return false;
    if ((a.x_ld * 2) % 16 || (a.K * a.bits / 8) % 16) return false;
    if (a.M > ((int64_t)1 << 31) - 1 || a.N > ((int64_t)1 << 31) - 1) return false;
    return encode_fn() != nullptr;
}

template <int BITS>
int launches_bits(const TcGemmArgs &a) {
    int64_t main_tiles = 0;
    int split = 1;
    if (a.M <= 64) plan_bm<BITS, 64>(a, &main_tiles, &split);
    else if (a.M <= 128) plan_bm<BITS, 128>(a, &main_tiles, &split);
    else plan_bm<BITS, 256>(a, &main_tiles, &split);
    return (main_tiles > 0 ? 1 : 0) + (split > 1 ? 1 : 0);
}

int tc_gemm_launches(const TcGemmArgs &a) {
    if (!tc_gemm_supported(a)) return 0;
    return a.bits == 4 ? launches_bits<4>(a) : launches_bits<8>(a);
}

template <bool F16>
cudaError_t launch_tc_dt(const TcGemmArgs &a, cudaStream_t stream) {
    if (a.M <= 64)
        return a.bits == 4 ? launch_bm<4, 64, F16>(a, stream) : launch_bm<8, 64, F16>(a, stream);
    if (a.M <= 128)
        return a.bits == 4 ? launch_bm<4, 128, F16>(a, stream) : launch_bm<8, 128, F16>(a, stream);
    return a.bits == 4 ? launch_bm<4, 256, F16>(a, stream) : launch_bm<8, 256, F16>(a, stream);
}

cudaError_t launch_tc_gemm(const TcGemmArgs &a, cudaStream_t stream) {
    if (!tc_gemm_supported(a)) return cudaErrorNotSupported;
    if (a.f16 && a.push) return cudaErrorNotSupported;  // the fan-out is bf16 only
    return a.f16 ? launch_tc_dt<true>(a, stream) : launch_tc_dt<false>(a, stream);
}

}  // namespace nq
