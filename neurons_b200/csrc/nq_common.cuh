// nq_common.cuh -- device-side helpers shared by the sm_100a kernels:
// bf16 packing, bounded mbarrier waits, single-CTA TMA loads and the
// tcgen05 (TMEM / UMMA) instruction wrappers.  Inline PTX only; no library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nq {

// Error word bits written by kernels.
enum DeviceError : unsigned int {
    kErrWaitTimeout = 1u,      // an mbarrier wait exceeded its time limit
    kErrBadIndex = 2u,         // a gather index was out of range
};

// Upper bound on any spin-wait inside a kernel, in nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ bf16x2

__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// (lo, hi) fp32 -> packed bf16x2 (lo in the low half), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// (a & mask) | orv in one lop3
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
    return d;
}

__device__ __forceinline__ uint16_t bf16_bits(__nv_bfloat16 h) {
    return *reinterpret_cast<uint16_t *>(&h);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
    return bf16_bits(__float2bfloat16_rn(f));
}

// Per-group dequantization constants for the packed-pair paths.
//   4-bit: t = bf16x2(128+q_a, 128+q_b) (exact);  fma(t, s, -128 s) computes
//   the exact product s*q and rounds it once = bf16(s*q); add.rn then gives
//   bf16(bf16(s*q) + b) -- the MLX CPU dequantized value bit for bit (the sum
//   of two bf16 values is exact in fp32 whenever it can round differently).
struct Dq4 {
    uint32_t s2, n2, b2;  // (s,s), (-128s,-128s), (b,b) as bf16x2
};

__device__ __forceinline__ Dq4 make_dq4(uint16_t s, uint16_t b) {
    Dq4 d;
    d.s2 = (uint32_t)s | ((uint32_t)s << 16);
    d.b2 = (uint32_t)b | ((uint32_t)b << 16);
    const uint32_t m128 = 0xC300C300u;  // (-128, -128)
    const uint32_t z = 0x80008000u;     // (-0, -0)
    d.n2 = bf2_fma(d.s2, m128, z);      // exact -128*s
    return d;
}

// pair j of a 4-bit word: (q_j, q_{j+4}) biased to bf16 128+q
__device__ __forceinline__ uint32_t q4_pair_biased(uint32_t w, int j) {
    return lop3_and_or(w >> (4 * j), 0x000F000Fu, 0x43004300u);
}

__device__ __forceinline__ uint32_t dq4_pair(uint32_t t, const Dq4 &d) {
    return bf2_add(bf2_fma(t, d.s2, d.n2), d.b2);
}

// 8-bit codes: byte -> fp32 2^23+q via prmt; fma with -2^23*s gives s*q
// exactly in fp32; cvt rounds it once to bf16; add.rn adds the bias.
struct Dq8 {
    float s, n;     // s, -2^23*s
    uint32_t b2;    // (b,b)
};

__device__ __forceinline__ Dq8 make_dq8(uint16_t s, uint16_t b) {
    Dq8 d;
    d.s = bf16_to_f32(s);
    d.n = -8388608.0f * d.s;
    d.b2 = (uint32_t)b | ((uint32_t)b << 16);
    return d;
}

// bytes i0, i1 of w -> dequantized bf16x2 (lo = code i0, hi = code i1)
__device__ __forceinline__ uint32_t dq8_pair(uint32_t w, int i0, int i1, const Dq8 &d) {
    const uint32_t magic = 0x4B000000u;  // byte0 <- w.byte[i], bytes1,2 <- 0, byte3 <- 0x4B
    const uint32_t fa = prmt(w, magic, 0x7440u | (uint32_t)i0);
    const uint32_t fb = prmt(w, magic, 0x7440u | (uint32_t)i1);
    const float pa = __fmaf_rn(__uint_as_float(fa), d.s, d.n);
    const float pb = __fmaf_rn(__uint_as_float(fb), d.s, d.n);
    return bf2_add(pack_bf2(pa, pb), d.b2);
}

// ------------------------------------------------------------------ fp16x2
// The same exact dequantization for fp16 scales and biases (fp16 checkpoints):
//   t = fp16x2(1024+q_a, 1024+q_b) (exact for q < 1024), t - 1024 = q exactly,
//   mul.rn(q, s) = fp16(s*q) (one rounding of the exact product), add.rn(., b)
//   = fp16(fp16(s*q) + b) -- MLX's dequantized fp16 value bit for bit.

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t h2_add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint16_t f32_to_f16(float f) {
    const __half h = __float2half_rn(f);
    return *reinterpret_cast<const uint16_t *>(&h);
}

__device__ __forceinline__ float f16_to_f32(uint16_t h) {
    return __half2float(*reinterpret_cast<const __half *>(&h));
}

// 16-bit storage type T of activations, scales and biases: bf16 or fp16
template <bool F16>
__device__ __forceinline__ uint16_t f32_to_t16(float f) {
    if constexpr (F16) return f32_to_f16(f);
    else return f32_to_bf16(f);
}

template <bool F16>
__device__ __forceinline__ float t16_to_f32(uint16_t h) {
    if constexpr (F16) return f16_to_f32(h);
    else return bf16_to_f32(h);
}

template <bool F16>
__device__ __forceinline__ uint32_t pack_t2(float lo, float hi) {
    if constexpr (F16) {
        uint32_t d;
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
        return d;
    } else {
        return pack_bf2(lo, hi);
    }
}

struct Dq4h {
    uint32_t s2, b2;  // (s,s), (b,b) as fp16x2
};

__device__ __forceinline__ Dq4h make_dq4h(uint16_t s, uint16_t b) {
    Dq4h d;
    d.s2 = (uint32_t)s | ((uint32_t)s << 16);
    d.b2 = (uint32_t)b | ((uint32_t)b << 16);
    return d;
}

// biased codes t = (1024 + q_a, 1024 + q_b) -> dequantized fp16x2
__device__ __forceinline__ uint32_t dqh_pair(uint32_t t, const Dq4h &d) {
    return h2_add(h2_mul(h2_sub(t, 0x64006400u), d.s2), d.b2);
}

// pair j of a 4-bit word: (q_j, q_{j+4}) biased to fp16 1024+q
__device__ __forceinline__ uint32_t q4_pair_biased_h(uint32_t w, int j) {
    return lop3_and_or(w >> (4 * j), 0x000F000Fu, 0x64006400u);
}

// bytes i0, i1 of w -> biased fp16x2 (1024 + byte)
__device__ __forceinline__ uint32_t q8_pair_biased_h(uint32_t w, int i0, int i1) {
    return prmt(w, 0x64646464u, (uint32_t)i0 | 0x40u | ((uint32_t)i1 << 8) | 0x4000u);
}

// --------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_load_2d(void *smem_dst, const void *tmap, uint64_t *bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory, completing on an
// mbarrier (no multicast).  Both addresses 16-byte aligned, bytes a multiple
// of 16.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(smem_dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// TMA store of a 2-D box from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const void *tmap, const void *smem_src, int32_t c0,
                                             int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
        "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until the committed bulk stores have read their shared-memory source.
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols));
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr),
                 "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (bf16 in, fp32 accumulate).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
            d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// Signals `bar` once every tcgen05.mma issued so far by this thread completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "
        "%10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]));
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte-swizzled canonical layout (8-row x 128-byte swizzle atoms, atoms
// 1024 bytes apart along M/N).  Bits: start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version=1 [46,48), layout SWIZZLE_128B=2 [61,64).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;              // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;    // SBO = 1024 B between 8-row groups
    d |= (uint64_t)1u << 46;              // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;              // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: fp16 A/B (format 0), fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int mma_m, int mma_n) {
    return (1u << 4)                              // D format f32
           | ((uint32_t)(mma_n >> 3) << 17)       // N >> 3
           | ((uint32_t)(mma_m >> 4) << 24);      // M >> 4
}

// Instruction descriptor, kind::f16: bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int mma_m, int mma_n) {
    return (1u << 4)                              // D format f32
           | (1u << 7)                            // A format bf16
           | (1u << 10)                           // B format bf16
           | ((uint32_t)(mma_n >> 3) << 17)       // N >> 3
           | ((uint32_t)(mma_m >> 4) << 24);      // M >> 4
}

// Bounded wait on an mbarrier phase shared by the roles of one CTA.  Gives up
// when another role raised *abort, or after kWaitLimitNs: then it raises
// *abort and the timeout bit of the device error word.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t *bar, uint32_t parity,
                                                   volatile int *abort, unsigned int *err) {
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

// 16-byte cp.async global -> shared (L2 only); src_bytes 0 writes zeros.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (tcgen05.mma operands, TMA stores).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Named barrier over `count` threads (a multiple of 32).
__device__ __forceinline__ void bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---------------------------------------------- tensor-parallel output push
// A kernel that computes one rank's column shard of y can write it straight
// into every rank's y (peer memory mapped with CUDA IPC) instead of handing
// it to an all-gather.  Per call number `epoch` (the same on every rank,
// increasing; in device memory, advanced by the ready kernel, so a CUDA graph
// of the calls stays correct on every replay):
//   * before the call, every rank's ready kernel sets ready[rank] = epoch in
//     every rank's memory (its stream's earlier work, which may still read
//     the buffers being written, has completed);
//   * a storing warp waits until all `ready` flags reached epoch, then stores
//     each value once per rank;
//   * after the kernel, a finish kernel (which the compute grid's completion
//     -- all its stores performed -- releases) publishes done[rank] = epoch
//     to every rank and waits for every rank's done flag.
// Every wait is bounded (kWaitLimitNs) and raises the timeout bit.
constexpr int kMaxRanks = 8;

struct PushDev {
    int n = 0;                           // ranks written; 0: plain local stores
    const unsigned *epoch = nullptr;     // this call's number (device memory)
    long long delta[kMaxRanks];          // bytes from the local y element to rank q's copy
    const unsigned *ready = nullptr;     // this rank's ready flags [n]
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Lane 0 of the calling warp waits for every rank's ready flag; false on timeout.
__device__ __forceinline__ bool push_wait_ready(const PushDev &p, unsigned int *err) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) {
        const unsigned long long t0 = global_timer_ns();
        const unsigned epoch = *p.epoch;
        for (int q = 0; q < p.n && ok; ++q) {
            while ((int)(ld_acquire_sys(p.ready + q) - epoch) < 0) {
                if (global_timer_ns() - t0 > kWaitLimitNs) {
                    atomicOr(err, kErrWaitTimeout);
                    ok = false;
                    break;
                }
            }
        }
    }
    return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

template <typename T>
__device__ __forceinline__ void push_store(const PushDev &p, T *local, T v) {
    if (p.n == 0) {
        *local = v;
        return;
    }
    for (int q = 0; q < p.n; ++q)
        *reinterpret_cast<T *>(reinterpret_cast<char *>(local) + p.delta[q]) = v;
}

// Programmatic dependent launch: wait for the producing grid / let the next
// grid start its prologue.  Both are no-ops without the launch attribute.
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;");
}

}  // namespace nq

namespace nq {

// ------------------------------------------- CTA pairs (cta_group::2 tcgen05)
// A cluster of two CTAs on two SMs shares one MMA: 256 weight rows (128 from
// each CTA's shared memory), N tokens (N/2 from each), accumulators in each
// CTA's TMEM.  One thread of the even CTA issues the MMAs.

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of `local` (this CTA's shared memory) in CTA `rank`'s shared memory,
// in the shared::cluster window.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}

// Arrive on an mbarrier in another CTA of the cluster (release at CTA scope,
// the form cluster pipelines use: a cluster-scope release measured ~0.8 us
// per arrival, blocking the issuing thread).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}

// Test (without suspending) with acquire at cluster scope: the phase may be
// completed by arrivals from the peer CTA, which -- measured -- do not wake a
// thread suspended in mbarrier.try_wait promptly (microseconds late), so
// the waiter polls.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols));
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr),
                 "r"(ncols));
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T over the CTA pair, kind::f16.
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, "
        "p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u));
}

// Once every tcgen05.mma issued so far by this thread completed, arrive on
// the mbarrier at this offset in each CTA of `cta_mask`.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
        "[%0], %1;" ::"r"(smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

}  // namespace nq
