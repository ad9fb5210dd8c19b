// dist.cu -- libnq_dist.so: tensor- and expert-parallel sharding of the
// quantized-matmul path over NCCL (one process per GPU).  Compute goes
// through libnq's C ABI (nq.h); this file adds the communicator, the
// collectives around the compute and two small layout kernels.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>

#include "nq.h"
#include "nq_dist.h"

// Symmetric arena: the same number of bytes on every rank, mapped into every
// other rank's address space with CUDA IPC.  A 4 KB header holds the flags of
// the fused tensor-parallel calls; the rest is for the callers' outputs.
//   ready[8] @ 0, done[8] @ 128, error word of the finish kernel @ 384
constexpr size_t kArenaHeader = 4096;
//   epoch (the fused calls made, advanced by the ready kernel) @ 448
//   table of the ready-flag addresses this rank writes (one per rank) @ 512
//   table of the done-flag addresses this rank writes (one per rank) @ 640
//   expert-parallel flags: dispatched[8] @ 1024, combined[8] @ 1152, and the
//   tables of the addresses this rank writes them to @ 1280 and @ 1408
constexpr size_t kReadyOff = 0, kDoneOff = 128, kErrOff = 384,
                 kEpochOff = 448, kTableOff = 512, kDoneTableOff = 640,
                 kDispOff = 1024, kCombOff = 1152, kDispTableOff = 1280, kCombTableOff = 1408;
// bits of the arena's error word
constexpr unsigned kCommErrTimeout = 1u;

struct nq_comm_s {
    ncclComm_t nccl = nullptr;
    int rank = 0;
    int size = 1;
    int device = 0;
    char *arena = nullptr;                 // this rank's arena (header + data)
    size_t arena_bytes = 0;                // data bytes
    char *peer[NQ_MAX_RANKS] = {};         // every rank's arena in this process (self included)
    int64_t timeout_ms = 0;                // > 0: every sharded call ends with nq_comm_wait
    bool aborted = false;                  // the NCCL communicator was aborted
};

namespace {

thread_local std::string g_err;

int fail(int status, const std::string &msg) {
    g_err = msg;
    return status;
}

int from_nq(int rc, const char *what) {
    if (rc == NQ_SUCCESS) return rc;
    const char *m = nq_last_error();
    g_err = std::string(what) + ": " + (m ? m : "");
    return rc;
}

int from_nccl(ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return NQ_SUCCESS;
    g_err = std::string(what) + ": NCCL: " + ncclGetErrorString(r);
    return NQ_COMPUTE_ERROR;
}

int from_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return NQ_SUCCESS;
    g_err = std::string(what) + ": CUDA: " + cudaGetErrorString(e);
    return NQ_COMPUTE_ERROR;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

int split(int64_t n, int nranks, int rank, int64_t *first, int64_t *count, const char *what) {
    if (nranks <= 0 || rank < 0 || rank >= nranks || n <= 0)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": need n > 0 and 0 <= rank < nranks");
    if (n % nranks)
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": " + std::to_string(n) + " is not a multiple of " +
                        std::to_string(nranks) + " ranks");
    if (!first || !count) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL output");
    *count = n / nranks;
    *first = (int64_t)rank * (*count);
    return NQ_SUCCESS;
}

// y[m, p * cols + j] = g[p][m][j]  (rank-major all-gather result -> row-major).
// One CTA per (p, m) run of cols elements, moved in 16-byte pieces when the
// run and both buffers allow it (cols % 8 == 0 and 16-byte aligned bases).
__global__ void rank_major_to_rows(const uint16_t *__restrict__ g, int64_t M, int64_t cols,
                                   int P, uint16_t *__restrict__ y, int vec) {
    for (int64_t run = blockIdx.x; run < (int64_t)P * M; run += gridDim.x) {
        const int64_t p = run / M, m = run % M;
        const uint16_t *src = g + run * cols;
        uint16_t *dst = y + m * cols * P + p * cols;
        if (vec) {
            const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
            uint4 *d4 = reinterpret_cast<uint4 *>(dst);
            for (int64_t j = threadIdx.x; j < cols / 8; j += blockDim.x) d4[j] = s4[j];
        } else {
            for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) dst[j] = src[j];
        }
    }
}

// y = bf16(v), round to nearest even
__global__ void f32_to_bf16_kernel(const float *__restrict__ v, int64_t n,
                                   uint16_t *__restrict__ y) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const __nv_bfloat16 b = __float2bfloat16_rn(v[i]);
        y[i] = *reinterpret_cast<const uint16_t *>(&b);
    }
}

struct EpWorkspace {
    uint16_t *x_all;
    int32_t *idx_all;
    float *sc_all;
    float *partial;
    float *mine;
    void *local;
    size_t local_bytes;
    size_t bytes;
};

EpWorkspace ep_carve(void *base, int64_t T, int64_t E, int64_t top_k, int64_t H, int64_t I,
                     int nranks) {
    EpWorkspace w{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = static_cast<char *>(base) + off;
        off += align256(bytes);
        return p;
    };
    w.x_all = reinterpret_cast<uint16_t *>(take(sizeof(uint16_t) * T * H));
    w.idx_all = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * T * top_k));
    w.sc_all = reinterpret_cast<float *>(take(sizeof(float) * T * top_k));
    w.partial = reinterpret_cast<float *>(take(sizeof(float) * T * H));
    w.mine = reinterpret_cast<float *>(take(sizeof(float) * (T / nranks) * H));
    w.local_bytes = nq_moe_partial_workspace_size(T, E, E / nranks, top_k, H, I);
    w.local = take(w.local_bytes);
    w.bytes = off;
    return w;
}

// Advances the call number and sets this rank's ready flag to it in every
// rank's arena, once the stream's earlier work has completed.  Launched as a
// programmatic dependent: the compute kernel after it may start (and fetch
// its weights) at once; it reads the flags only after its own
// griddepcontrol.wait, i.e. after this kernel completed.
__global__ void push_ready_kernel(unsigned int *const *flags, int n, unsigned int *epoch) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int q = threadIdx.x;
    const unsigned int e = *epoch + 1;
    __syncwarp();
    if (q == 0) *epoch = e;
    if (q < n) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags[q]), "r"(e)
                            : "memory");
}

// After the compute grid (whose completion, awaited by griddepcontrol.wait,
// means all its stores -- peer stores included -- are performed): publish
// this rank's done flag to every rank, then wait (bounded) until every rank's
// done flag here reached the call number.  When this kernel completes, every
// rank's columns are in this rank's y.
__global__ void push_finish_kernel(unsigned int *const *done_remote, const unsigned int *done_local,
                                   int n, const unsigned int *epoch_p, unsigned int *err) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int q = threadIdx.x;
    const unsigned int epoch = *epoch_p;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    if (q < n)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(done_remote[q]), "r"(epoch)
                     : "memory");
    if (q >= n) return;
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (true) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(done_local + q)
                     : "memory");
        if ((int)(v - epoch) >= 0) return;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > 2000000000ull) {
            atomicOr(err, 1u);
            return;
        }
    }
}

cudaError_t launch_pdl_1warp(cudaStream_t st, void (*kern)(unsigned int *const *, const unsigned int *, int, const unsigned int *, unsigned int *),
                             unsigned int *const *a, const unsigned int *b, int n,
                             const unsigned int *e, unsigned int *err) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, b, n, e, err);
}

// ---------------------------------------------------------------------------
// Expert-parallel switch step with an all-to-all over peer memory.
//
// Rank r owns tokens [r * cap, (r + 1) * cap) (cap = T / P) and experts
// [r * ne, (r + 1) * ne).  Each rank's EP region of the arena holds, for every
// source rank q, the token rows q sent it and the partial results it gets back:
//   recv_x   [P][cap][H] bf16    token rows, region q written by rank q
//   recv_idx [P][cap][k] int32   their routing (all k slots, as routed)
//   recv_sc  [P][cap][k] fp32
//   recv_cnt [P]        int32    rows rank q sent (written by rank q)
//   back     [P][cap][H] fp32    region d: rank d's partial sums for this
//                                rank's tokens, at the rows this rank chose
// A token goes once to every rank that holds at least one of its experts.
// ---------------------------------------------------------------------------
struct EpRegion {
    size_t x = 0, idx = 0, sc = 0, cnt = 0, back = 0, bytes = 0;
};

EpRegion ep_region(int64_t cap, int64_t k, int64_t H, int P) {
    EpRegion g;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += align256(bytes);
        return at;
    };
    g.x = take(sizeof(uint16_t) * P * cap * H);
    g.idx = take(sizeof(int32_t) * P * cap * k);
    g.sc = take(sizeof(float) * P * cap * k);
    g.cnt = take(sizeof(int32_t) * P);
    g.back = take(sizeof(float) * P * cap * H);
    g.bytes = off;
    return g;
}

struct EpPeers {
    char *region[NQ_MAX_RANKS];  // every rank's EP region, mapped in this process
};

// this rank's local scratch: pos[cap][P] (row of token t in rank q's region q
// of recv_x, -1: not sent), send_cnt[P], then the shard's switch workspace
struct EpLocal {
    int32_t *pos = nullptr, *send_cnt = nullptr;
    void *sw = nullptr;
    size_t sw_bytes = 0, bytes = 0;
};

EpLocal ep_local(void *base, int64_t T, int64_t E, int64_t k, int64_t H, int64_t I, int P) {
    EpLocal l;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = static_cast<char *>(base) + off;
        off += align256(bytes);
        return p;
    };
    l.pos = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * (T / P) * P));
    l.send_cnt = reinterpret_cast<int32_t *>(take(sizeof(int32_t) * P));
    l.sw_bytes = nq_moe_partial_workspace_size(T, E, E / P, k, H, I);
    l.sw = take(l.sw_bytes);
    l.bytes = off;
    return l;
}

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait until flag >= epoch (wrapping compare); false on timeout.
__device__ bool wait_flag(const unsigned *flag, unsigned epoch, unsigned *err) {
    const unsigned long long t0 = timer_ns();
    while ((int)(ld_acquire_sys_u32(flag) - epoch) < 0) {
        if (timer_ns() - t0 > 2000000000ull) {
            atomicOr(err, kCommErrTimeout);
            return false;
        }
    }
    return true;
}

// Dispatch: one warp per local token.  After every rank's ready flag reached
// this call's number (their earlier calls no longer read their regions), the
// token's destinations are the ranks of its valid slots; each takes the next
// row of its region for this rank (atomic counter, so rows are in no fixed
// order -- every row is computed on its own, so results do not depend on it),
// and the warp writes the token's x row (16-byte stores) and routing there.
__global__ void ep_dispatch_kernel(const uint16_t *__restrict__ x, const int32_t *__restrict__ idx,
                                   const float *__restrict__ sc, int64_t cap, int64_t H, int k,
                                   int E, int ne, int P, int rank, EpPeers peers, EpRegion rg,
                                   int32_t *send_cnt, int32_t *pos, const unsigned *ready,
                                   const unsigned *epoch_p, unsigned *err) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    if (warp >= cap) return;
    int ok = 1;
    if (lane == 0) {
        const unsigned epoch = *epoch_p;
        for (int q = 0; q < P && ok; ++q) ok = wait_flag(ready + q, epoch, err);
    }
    if (!__shfl_sync(0xffffffffu, ok, 0)) return;
    for (int64_t t = warp; t < cap; t += nwarps) {
        const int e = lane < k ? idx[t * k + lane] : -1;
        const float s = lane < k ? sc[t * k + lane] : 0.f;
        const bool valid = lane < k && e >= 0 && e < E;
        const unsigned mask = __reduce_or_sync(0xffffffffu, valid ? 1u << (e / ne) : 0u);
        int p = -1;
        if (lane < P && ((mask >> lane) & 1u)) p = atomicAdd(&send_cnt[lane], 1);
        if (lane < P) pos[t * P + lane] = p;
        const uint4 *src = reinterpret_cast<const uint4 *>(x + t * H);
        for (int q = 0; q < P; ++q) {
            const int pq = __shfl_sync(0xffffffffu, p, q);
            if (pq < 0) continue;
            const int64_t row = (int64_t)rank * cap + pq;
            uint4 *dx = reinterpret_cast<uint4 *>(peers.region[q] + rg.x) + row * (H / 8);
            for (int64_t j = lane; j < H / 8; j += 32) dx[j] = src[j];
            if (lane < k) {
                // an out-of-range expert is passed on as it is: the receiver's
                // switch step flags it in the device error word and skips it
                reinterpret_cast<int32_t *>(peers.region[q] + rg.idx)[row * k + lane] = e;
                reinterpret_cast<float *>(peers.region[q] + rg.sc)[row * k + lane] = s;
            }
        }
    }
}

// After the dispatch grid: send every rank the number of rows written into
// its region for this rank, publish this rank's dispatched flag everywhere,
// wait (bounded) for every rank's, then mark the unused rows of every region
// of this rank's own EP region as routed to e_pad with score 0 (an expert of
// another rank, or with one rank a zero-weight slot) so that the switch step
// skips or discards them.
__global__ void ep_exchange_kernel(EpPeers peers, EpRegion rg, int P, int rank, int64_t cap, int k,
                                   int e_pad, const int32_t *send_cnt,
                                   unsigned int *const *disp_remote, const unsigned *disp_local,
                                   const unsigned *epoch_p, unsigned *err) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ int ok;
    const int q = threadIdx.x;
    const unsigned epoch = *epoch_p;
    if (q == 0) ok = 1;
    if (q < P) reinterpret_cast<int32_t *>(peers.region[q] + rg.cnt)[rank] = send_cnt[q];
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    if (q < P)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(disp_remote[q]), "r"(epoch)
                     : "memory");
    __syncthreads();
    if (q < P && !wait_flag(disp_local + q, epoch, err)) ok = 0;
    __syncthreads();
    if (!ok) return;
    char *mine = peers.region[rank];
    const int32_t *cnt = reinterpret_cast<const int32_t *>(mine + rg.cnt);
    int32_t *ridx = reinterpret_cast<int32_t *>(mine + rg.idx);
    float *rsc = reinterpret_cast<float *>(mine + rg.sc);
    const int64_t n = (int64_t)P * cap * k;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const int64_t row = i / k;
        if (row % cap >= cnt[row / cap]) {
            ridx[i] = e_pad;
            rsc[i] = 0.f;
        }
    }
}

// y[t] = bf16(sum over ranks d = 0..P-1 that computed for token t of their
// partial sums), in that order.
__global__ void ep_final_kernel(const float *__restrict__ back, const int32_t *__restrict__ pos,
                                int64_t cap, int64_t H, int P, uint16_t *__restrict__ y) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over cap * H / 4
    if (i >= cap * (H / 4)) return;
    const int64_t t = i / (H / 4), n = (i % (H / 4)) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d < P; ++d) {
        const int p = pos[t * P + d];
        if (p < 0) continue;
        const float4 v = *reinterpret_cast<const float4 *>(back + ((int64_t)d * cap + p) * H + n);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t *>(&lo);
    o.y = *reinterpret_cast<const uint32_t *>(&hi);
    *reinterpret_cast<uint2 *>(y + t * H + n) = o;
}

template <typename... Args>
cudaError_t launch_pdl_k(void (*kern)(Args...), unsigned blocks, unsigned threads, cudaStream_t st,
                         Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(threads);
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

unsigned grid_for(int64_t n) {
    const int64_t b = (n + 255) / 256;
    return (unsigned)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

}  // namespace

extern "C" int nq_comm_wait(nq_comm_t comm, void *stream, int64_t timeout_ms);

namespace {
// A sharded call that succeeded ends with the communicator's bounded wait
// when one is set (nq_comm_set_timeout).
int settle(nq_comm_t comm, void *stream, int rc) {
    if (rc != NQ_SUCCESS || !comm || comm->timeout_ms <= 0) return rc;
    return nq_comm_wait(comm, stream, comm->timeout_ms);
}
}  // namespace

extern "C" {

const char *nq_dist_last_error(void) { return g_err.c_str(); }

int nq_comm_unique_id(unsigned char id[NQ_COMM_ID_BYTES]) {
    if (!id) return fail(NQ_INVALID_INPUT, "nq_comm_unique_id: NULL id");
    ncclUniqueId u;
    if (int rc = from_nccl(ncclGetUniqueId(&u), "nq_comm_unique_id")) return rc;
    static_assert(sizeof(u) == NQ_COMM_ID_BYTES, "NCCL unique id size");
    std::memcpy(id, &u, sizeof(u));
    return NQ_SUCCESS;
}

int nq_comm_init(nq_comm_t *comm, int nranks, int rank, const unsigned char id[NQ_COMM_ID_BYTES]) {
    if (!comm || !id) return fail(NQ_INVALID_INPUT, "nq_comm_init: NULL argument");
    if (nranks <= 0 || rank < 0 || rank >= nranks)
        return fail(NQ_INVALID_INPUT, "nq_comm_init: need 0 <= rank < nranks");
    int dev = 0;
    if (int rc = from_cuda(cudaGetDevice(&dev), "nq_comm_init")) return rc;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    nq_comm_s *c = new nq_comm_s;
    c->rank = rank;
    c->size = nranks;
    c->device = dev;
    if (int rc = from_nccl(ncclCommInitRank(&c->nccl, nranks, u, rank), "nq_comm_init")) {
        delete c;
        return rc;
    }
    *comm = c;
    return NQ_SUCCESS;
}

static void release_arena(nq_comm_t comm) {
    for (int q = 0; q < comm->size; ++q)
        if (comm->peer[q] && q != comm->rank) cudaIpcCloseMemHandle(comm->peer[q]);
    if (comm->arena) cudaFree(comm->arena);
    comm->arena = nullptr;
    for (auto &p : comm->peer) p = nullptr;
}

int nq_comm_destroy(nq_comm_t comm) {
    if (!comm) return NQ_SUCCESS;
    release_arena(comm);
    const int rc =
        comm->aborted ? NQ_SUCCESS : from_nccl(ncclCommDestroy(comm->nccl), "nq_comm_destroy");
    delete comm;
    return rc;
}

int nq_comm_abort(nq_comm_t comm) {
    if (!comm) return NQ_SUCCESS;
    release_arena(comm);
    const int rc =
        comm->aborted ? NQ_SUCCESS : from_nccl(ncclCommAbort(comm->nccl), "nq_comm_abort");
    delete comm;
    return rc;
}

int nq_comm_set_timeout(nq_comm_t comm, int64_t timeout_ms) {
    if (!comm || timeout_ms < 0)
        return fail(NQ_INVALID_INPUT, "nq_comm_set_timeout: NULL communicator or negative timeout");
    comm->timeout_ms = timeout_ms;
    return NQ_SUCCESS;
}

int nq_comm_wait(nq_comm_t comm, void *stream, int64_t timeout_ms) {
    const char *what = "nq_comm_wait";
    if (!comm || timeout_ms <= 0)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL communicator or timeout <= 0");
    if (comm->aborted)
        return fail(NQ_COMPUTE_ERROR, std::string(what) + ": the communicator was aborted");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    using clock = std::chrono::steady_clock;
    const auto deadline = clock::now() + std::chrono::milliseconds(timeout_ms);
    std::string why;
    while (true) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return NQ_SUCCESS;
        if (q != cudaErrorNotReady) return from_cuda(q, what);
        ncclResult_t async = ncclSuccess;
        const ncclResult_t r = ncclCommGetAsyncError(comm->nccl, &async);
        if (r != ncclSuccess || (async != ncclSuccess && async != ncclInProgress)) {
            why = std::string("NCCL reported an error: ") +
                  ncclGetErrorString(r != ncclSuccess ? r : async);
            break;
        }
        if (clock::now() > deadline) {
            why = "timed out after " + std::to_string(timeout_ms) +
                  " ms (a rank left or stopped calling)";
            break;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
    // end the collectives still waiting, then let the stream drain (bounded)
    ncclCommAbort(comm->nccl);
    comm->aborted = true;
    const auto drain = clock::now() + std::chrono::seconds(10);
    while (cudaStreamQuery(st) == cudaErrorNotReady && clock::now() < drain)
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    const bool drained = cudaStreamQuery(st) != cudaErrorNotReady;
    cudaGetLastError();
    return fail(NQ_COMPUTE_ERROR, std::string(what) + ": " + why +
                                      "; communicator aborted" +
                                      (drained ? "" : ", stream still busy after 10 s"));
}

int nq_comm_rank(nq_comm_t comm) { return comm ? comm->rank : -1; }
int nq_comm_size(nq_comm_t comm) { return comm ? comm->size : -1; }

int nq_comm_symmetric_alloc(nq_comm_t comm, size_t bytes) {
    const char *what = "nq_comm_symmetric_alloc";
    if (!comm) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL communicator");
    if (comm->arena) return fail(NQ_INVALID_INPUT, std::string(what) + ": already allocated");
    if (comm->size > NQ_MAX_RANKS)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": more than 8 ranks");
    bytes = (bytes + 255) & ~size_t(255);
    char *base = nullptr;
    if (int rc = from_cuda(cudaMalloc(&base, kArenaHeader + bytes), what)) return rc;
    cudaIpcMemHandle_t *all = nullptr;
    cudaIpcMemHandle_t mine;
    int rc = from_cuda(cudaMemset(base, 0, kArenaHeader + bytes), what);
    if (!rc) rc = from_cuda(cudaIpcGetMemHandle(&mine, base), what);
    // every rank's handle, through the communicator
    void *dev = nullptr;
    if (!rc) rc = from_cuda(cudaMalloc(&dev, sizeof(cudaIpcMemHandle_t) * comm->size), what);
    if (!rc) rc = from_cuda(cudaMemcpy(static_cast<char *>(dev) + sizeof(mine) * comm->rank, &mine,
                                       sizeof(mine), cudaMemcpyHostToDevice),
                            what);
    if (!rc) rc = from_nccl(ncclAllGather(static_cast<char *>(dev) + sizeof(mine) * comm->rank, dev,
                                          sizeof(mine), ncclUint8, comm->nccl, nullptr),
                            what);
    if (!rc) rc = from_cuda(cudaDeviceSynchronize(), what);
    if (!rc) {
        all = new cudaIpcMemHandle_t[comm->size];
        rc = from_cuda(cudaMemcpy(all, dev, sizeof(mine) * comm->size, cudaMemcpyDeviceToHost), what);
    }
    if (dev) cudaFree(dev);
    comm->arena = base;
    comm->arena_bytes = bytes;
    for (int q = 0; !rc && q < comm->size; ++q) {
        if (q == comm->rank) {
            comm->peer[q] = base;
            continue;
        }
        void *p = nullptr;
        rc = from_cuda(cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess), what);
        comm->peer[q] = static_cast<char *>(p);
    }
    delete[] all;
    if (!rc) {
        unsigned int *ready_dst[NQ_MAX_RANKS];
        for (int q = 0; q < comm->size; ++q)
            ready_dst[q] = reinterpret_cast<unsigned int *>(comm->peer[q] + kReadyOff) + comm->rank;
        rc = from_cuda(cudaMemcpy(base + kTableOff, ready_dst, sizeof(void *) * comm->size,
                                  cudaMemcpyHostToDevice),
                       what);
        unsigned int *done_dst[NQ_MAX_RANKS];
        for (int q = 0; q < comm->size; ++q)
            done_dst[q] = reinterpret_cast<unsigned int *>(comm->peer[q] + kDoneOff) + comm->rank;
        if (!rc)
            rc = from_cuda(cudaMemcpy(base + kDoneTableOff, done_dst, sizeof(void *) * comm->size,
                                      cudaMemcpyHostToDevice),
                           what);
        unsigned int *disp_dst[NQ_MAX_RANKS], *comb_dst[NQ_MAX_RANKS];
        for (int q = 0; q < comm->size; ++q) {
            disp_dst[q] = reinterpret_cast<unsigned int *>(comm->peer[q] + kDispOff) + comm->rank;
            comb_dst[q] = reinterpret_cast<unsigned int *>(comm->peer[q] + kCombOff) + comm->rank;
        }
        if (!rc)
            rc = from_cuda(cudaMemcpy(base + kDispTableOff, disp_dst, sizeof(void *) * comm->size,
                                      cudaMemcpyHostToDevice),
                           what);
        if (!rc)
            rc = from_cuda(cudaMemcpy(base + kCombTableOff, comb_dst, sizeof(void *) * comm->size,
                                      cudaMemcpyHostToDevice),
                           what);
    }
    if (rc) release_arena(comm);
    return rc;
}

void *nq_comm_symmetric_ptr(nq_comm_t comm, size_t offset) {
    if (!comm || !comm->arena || offset >= comm->arena_bytes) return nullptr;
    return comm->arena + kArenaHeader + offset;
}

int nq_comm_take_error(nq_comm_t comm, unsigned int *value) {
    if (!comm || !value) return fail(NQ_INVALID_INPUT, "nq_comm_take_error: NULL argument");
    *value = 0;
    if (!comm->arena) return NQ_SUCCESS;
    unsigned int zero = 0;
    if (int rc = from_cuda(cudaMemcpy(value, comm->arena + kErrOff, sizeof(unsigned int),
                                      cudaMemcpyDeviceToHost),
                           "nq_comm_take_error"))
        return rc;
    return from_cuda(cudaMemcpy(comm->arena + kErrOff, &zero, sizeof(zero), cudaMemcpyHostToDevice),
                     "nq_comm_take_error");
}

static int tp_quantized_matmul_fused_impl(nq_comm_t comm, const uint16_t *x, int64_t M,
                                 const uint32_t *w_shard, const uint16_t *s_shard,
                                 const uint16_t *b_shard, int64_t N, int64_t K, int bits,
                                 int group_size, uint16_t *y, void *stream) {
    const char *what = "nq_tp_quantized_matmul_fused";
    if (!comm) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL communicator");
    if (!comm->arena)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": call nq_comm_symmetric_alloc first");
    int64_t row0, rows;
    if (int rc = split(N, comm->size, comm->rank, &row0, &rows, what)) return rc;
    if (M <= 0) return fail(NQ_INVALID_INPUT, std::string(what) + ": M must be > 0");
    char *data = comm->arena + kArenaHeader;
    const char *yc = reinterpret_cast<const char *>(y);
    if (yc < data || yc + (size_t)M * N * sizeof(uint16_t) > data + comm->arena_bytes ||
        (reinterpret_cast<uintptr_t>(y) & 15))
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": y must lie in the symmetric arena, 16-byte aligned");
    const size_t off = (size_t)(yc - data);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned int *epoch = reinterpret_cast<unsigned int *>(comm->arena + kEpochOff);
    nq_push_t p;
    std::memset(&p, 0, sizeof(p));
    p.nranks = comm->size;
    p.rank = comm->rank;
    p.epoch = epoch;
    p.ready = reinterpret_cast<const unsigned int *>(comm->arena + kReadyOff);
    for (int q = 0; q < comm->size; ++q) p.dst[q] = comm->peer[q] + kArenaHeader + off;
    // Every check of the compute step runs before anything is enqueued: a
    // rejected call launches nothing and leaves the call count (the epoch)
    // where it was.  (A rejection on some ranks only leaves the others' calls
    // to end on their bounded waits, with the timeout bit set.)
    if (int rc = from_nq(nq_quantized_matmul_push_check(x, M, w_shard, s_shard, b_shard, rows, K,
                                                        bits, group_size, N, row0, &p),
                         what))
        return rc;
    // ready: this rank's earlier stream work is done; tell every rank
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1);
        cfg.blockDim = dim3(32);
        cfg.stream = st;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr.val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (int rc = from_cuda(
                cudaLaunchKernelEx(&cfg, push_ready_kernel,
                                   reinterpret_cast<unsigned int *const *>(comm->arena + kTableOff),
                                   comm->size, epoch),
                what))
            return rc;
    }
    if (int rc = from_nq(nq_quantized_matmul_push(x, M, w_shard, s_shard, b_shard, rows, K, bits,
                                                  group_size, N, row0, &p, stream),
                         what))
        return rc;
    return from_cuda(
        launch_pdl_1warp(st, push_finish_kernel,
                         reinterpret_cast<unsigned int *const *>(comm->arena + kDoneTableOff),
                         reinterpret_cast<const unsigned int *>(comm->arena + kDoneOff),
                         comm->size, epoch, reinterpret_cast<unsigned int *>(comm->arena + kErrOff)),
        what);
}

int nq_tp_quantized_matmul_fused(nq_comm_t comm, const uint16_t *x, int64_t M,
                                 const uint32_t *w_shard, const uint16_t *s_shard,
                                 const uint16_t *b_shard, int64_t N, int64_t K, int bits,
                                 int group_size, uint16_t *y, void *stream) {
    if (comm && comm->aborted)
        return fail(NQ_COMPUTE_ERROR, "nq_tp_quantized_matmul_fused: the communicator was aborted");
    const int rc = tp_quantized_matmul_fused_impl(comm, x, M, w_shard, s_shard, b_shard, N, K, bits,
                                                  group_size, y, stream);
    return settle(comm, stream, rc);
}

int nq_tp_shard(int64_t N, int nranks, int rank, int64_t *row0, int64_t *rows) {
    return split(N, nranks, rank, row0, rows, "nq_tp_shard");
}

int nq_ep_shard(int64_t E, int nranks, int rank, int64_t *e0, int64_t *ne) {
    return split(E, nranks, rank, e0, ne, "nq_ep_shard");
}

int nq_ep_token_shard(int64_t T, int nranks, int rank, int64_t *t0, int64_t *nt) {
    return split(T, nranks, rank, t0, nt, "nq_ep_token_shard");
}

size_t nq_tp_workspace_size(int64_t M, int64_t N, int nranks) {
    if (M <= 1 || N <= 0 || nranks <= 0) return 0;
    return sizeof(uint16_t) * (size_t)M * (size_t)N;
}

size_t nq_ep_workspace_size(int64_t T, int64_t E, int64_t top_k, int64_t H, int64_t I,
                            int nranks) {
    if (T <= 0 || E <= 0 || top_k <= 0 || H <= 0 || I <= 0 || nranks <= 0) return 0;
    if (T % nranks || E % nranks) return 0;
    return ep_carve(nullptr, T, E, top_k, H, I, nranks).bytes;
}

static int tp_quantized_matmul_impl(nq_comm_t comm, const uint16_t *x, int64_t M, const uint32_t *w_shard,
                           const uint16_t *s_shard, const uint16_t *b_shard, int64_t N, int64_t K,
                           int bits, int group_size, uint16_t *y, void *workspace,
                           size_t workspace_bytes, void *stream) {
    const char *what = "nq_tp_quantized_matmul";
    if (!comm) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL communicator");
    int64_t row0, rows;
    if (int rc = split(N, comm->size, comm->rank, &row0, &rows, what)) return rc;
    if (M <= 0) return fail(NQ_INVALID_INPUT, std::string(what) + ": M must be > 0");
    if (!y) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL y");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int P = comm->size;
    if (M == 1) {
        // each rank's columns land in place; the all-gather fills the rest of y
        uint16_t *mine = y + row0;
        if (int rc = from_nq(nq_quantized_matmul(x, 1, w_shard, s_shard, b_shard, rows, K, bits,
                                                 group_size, mine, stream),
                             what))
            return rc;
        return from_nccl(ncclAllGather(mine, y, (size_t)rows, ncclBfloat16, comm->nccl, st), what);
    }
    const size_t need = nq_tp_workspace_size(M, N, P);
    if (!workspace || workspace_bytes < need)
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": workspace too small: need " + std::to_string(need));
    uint16_t *g = static_cast<uint16_t *>(workspace);  // [P][M][rows]
    uint16_t *mine = g + (size_t)comm->rank * M * rows;
    if (int rc = from_nq(nq_quantized_matmul(x, M, w_shard, s_shard, b_shard, rows, K, bits,
                                             group_size, mine, stream),
                         what))
        return rc;
    if (int rc = from_nccl(
            ncclAllGather(mine, g, (size_t)(M * rows), ncclBfloat16, comm->nccl, st), what))
        return rc;
    const int vec = rows % 8 == 0 && !(reinterpret_cast<uintptr_t>(g) & 15) &&
                    !(reinterpret_cast<uintptr_t>(y) & 15);
    const int64_t runs = (int64_t)P * M;
    rank_major_to_rows<<<(unsigned)std::min<int64_t>(runs, 148 * 8), 128, 0, st>>>(g, M, rows, P,
                                                                                   y, vec);
    return from_cuda(cudaGetLastError(), what);
}

int nq_tp_quantized_matmul(nq_comm_t comm, const uint16_t *x, int64_t M, const uint32_t *w_shard,
                           const uint16_t *s_shard, const uint16_t *b_shard, int64_t N, int64_t K,
                           int bits, int group_size, uint16_t *y, void *workspace,
                           size_t workspace_bytes, void *stream) {
    if (comm && comm->aborted)
        return fail(NQ_COMPUTE_ERROR, "nq_tp_quantized_matmul: the communicator was aborted");
    const int rc = tp_quantized_matmul_impl(comm, x, M, w_shard, s_shard, b_shard, N, K, bits,
                                            group_size, y, workspace, workspace_bytes, stream);
    return settle(comm, stream, rc);
}

static int ep_moe_switch_impl(nq_comm_t comm, const uint16_t *x_shard, int64_t T, int64_t H, int64_t I,
                     int64_t E, int64_t top_k, const int32_t *topk_idx_shard,
                     const float *topk_scores_shard, const uint32_t *gate_w,
                     const uint16_t *gate_s, const uint16_t *gate_b, const uint32_t *up_w,
                     const uint16_t *up_s, const uint16_t *up_b, const uint32_t *down_w,
                     const uint16_t *down_s, const uint16_t *down_b, int bits, int group_size,
                     void *workspace, size_t workspace_bytes, uint16_t *y_shard, void *stream) {
    const char *what = "nq_ep_moe_switch";
    if (!comm) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL communicator");
    int64_t e0, ne, t0, nt;
    if (int rc = split(E, comm->size, comm->rank, &e0, &ne, what)) return rc;
    if (int rc = split(T, comm->size, comm->rank, &t0, &nt, what)) return rc;
    if (!x_shard || !topk_idx_shard || !topk_scores_shard || !y_shard || !workspace)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL pointer");
    const size_t need = nq_ep_workspace_size(T, E, top_k, H, I, comm->size);
    if (need == 0 || workspace_bytes < need)
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": workspace too small: need " + std::to_string(need));
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": workspace must be 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    EpWorkspace w = ep_carve(workspace, T, E, top_k, H, I, comm->size);
    // dispatch: every rank gets every token and its routing
    if (int rc = from_nccl(ncclGroupStart(), what)) return rc;
    ncclAllGather(x_shard, w.x_all, (size_t)(nt * H), ncclBfloat16, comm->nccl, st);
    ncclAllGather(topk_idx_shard, w.idx_all, (size_t)(nt * top_k), ncclInt32, comm->nccl, st);
    ncclAllGather(topk_scores_shard, w.sc_all, (size_t)(nt * top_k), ncclFloat32, comm->nccl, st);
    if (int rc = from_nccl(ncclGroupEnd(), what)) return rc;
    // this rank's experts over all tokens
    if (int rc = from_nq(nq_moe_switch_partial(w.x_all, T, H, I, E, top_k, w.idx_all, w.sc_all,
                                               e0, ne, gate_w, gate_s, gate_b, up_w, up_s, up_b,
                                               down_w, down_s, down_b, bits, group_size, w.local,
                                               w.local_bytes, w.partial, stream),
                         what))
        return rc;
    // combine: sum the shards' partials, each rank keeps its own tokens
    if (int rc = from_nccl(ncclReduceScatter(w.partial, w.mine, (size_t)(nt * H), ncclFloat32,
                                             ncclSum, comm->nccl, st),
                           what))
        return rc;
    f32_to_bf16_kernel<<<grid_for(nt * H), 256, 0, st>>>(w.mine, nt * H, y_shard);
    return from_cuda(cudaGetLastError(), what);
}

int nq_ep_moe_switch(nq_comm_t comm, const uint16_t *x_shard, int64_t T, int64_t H, int64_t I,
                     int64_t E, int64_t top_k, const int32_t *topk_idx_shard,
                     const float *topk_scores_shard, const uint32_t *gate_w,
                     const uint16_t *gate_s, const uint16_t *gate_b, const uint32_t *up_w,
                     const uint16_t *up_s, const uint16_t *up_b, const uint32_t *down_w,
                     const uint16_t *down_s, const uint16_t *down_b, int bits, int group_size,
                     void *workspace, size_t workspace_bytes, uint16_t *y_shard, void *stream) {
    if (comm && comm->aborted)
        return fail(NQ_COMPUTE_ERROR, "nq_ep_moe_switch: the communicator was aborted");
    const int rc = ep_moe_switch_impl(comm, x_shard, T, H, I, E, top_k, topk_idx_shard,
                                      topk_scores_shard, gate_w, gate_s, gate_b, up_w, up_s, up_b,
                                      down_w, down_s, down_b, bits, group_size, workspace,
                                      workspace_bytes, y_shard, stream);
    return settle(comm, stream, rc);
}

size_t nq_ep_fused_arena_size(int64_t T, int64_t top_k, int64_t H, int nranks) {
    if (T <= 0 || top_k <= 0 || H <= 0 || nranks <= 0 || nranks > NQ_MAX_RANKS || T % nranks)
        return 0;
    return ep_region(T / nranks, top_k, H, nranks).bytes;
}

size_t nq_ep_fused_workspace_size(int64_t T, int64_t E, int64_t top_k, int64_t H, int64_t I,
                                  int nranks) {
    if (T <= 0 || E <= 0 || top_k <= 0 || H <= 0 || I <= 0 || nranks <= 0 ||
        nranks > NQ_MAX_RANKS || T % nranks || E % nranks)
        return 0;
    return ep_local(nullptr, T, E, top_k, H, I, nranks).bytes;
}

static int ep_moe_switch_fused_impl(nq_comm_t comm, const uint16_t *x_shard, int64_t T, int64_t H,
                           int64_t I, int64_t E, int64_t top_k, const int32_t *topk_idx_shard,
                           const float *topk_scores_shard, const uint32_t *gate_w,
                           const uint16_t *gate_s, const uint16_t *gate_b, const uint32_t *up_w,
                           const uint16_t *up_s, const uint16_t *up_b, const uint32_t *down_w,
                           const uint16_t *down_s, const uint16_t *down_b, int bits,
                           int group_size, size_t arena_offset, void *workspace,
                           size_t workspace_bytes, uint16_t *y_shard, void *stream) {
    const char *what = "nq_ep_moe_switch_fused";
    if (!comm) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL communicator");
    if (!comm->arena)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": call nq_comm_symmetric_alloc first");
    const int P = comm->size, rank = comm->rank;
    int64_t e0, ne, t0, cap;
    if (int rc = split(E, P, rank, &e0, &ne, what)) return rc;
    if (int rc = split(T, P, rank, &t0, &cap, what)) return rc;
    // Every check runs before anything is enqueued; with the same shapes on
    // every rank they agree, so no rank starts a call the others reject.
    if (!x_shard || !topk_idx_shard || !topk_scores_shard || !y_shard || !workspace || !gate_w ||
        !gate_s || !gate_b || !up_w || !up_s || !up_b || !down_w || !down_s || !down_b)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL pointer");
    if (top_k <= 0 || top_k > 32 || top_k > E || E > 1024 || H % 8 || H <= 0 || I <= 0)
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": need 0 < top_k <= min(E, 32), E <= 1024, H % 8 == 0");
    if ((bits != 4 && bits != 8) || (group_size != 32 && group_size != 64 && group_size != 128) ||
        H % group_size || I % group_size)
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": bits 4 or 8, group size 32/64/128 dividing H and I");
    const uintptr_t a16 = reinterpret_cast<uintptr_t>(x_shard) |
                          reinterpret_cast<uintptr_t>(y_shard) |
                          reinterpret_cast<uintptr_t>(gate_w) | reinterpret_cast<uintptr_t>(up_w) |
                          reinterpret_cast<uintptr_t>(down_w);
    if (a16 & 15)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": x, y and weights must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": workspace must be 256-byte aligned");
    const size_t need = nq_ep_fused_workspace_size(T, E, top_k, H, I, P);
    if (need == 0 || workspace_bytes < need)
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": workspace too small: need " + std::to_string(need));
    const EpRegion rg = ep_region(cap, top_k, H, P);
    if (arena_offset % 256 || arena_offset + rg.bytes > comm->arena_bytes)
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": the EP region (nq_ep_fused_arena_size bytes at a "
                                        "256-byte aligned offset) must lie in the arena");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    EpLocal loc = ep_local(workspace, T, E, top_k, H, I, P);
    EpPeers peers;
    for (int q = 0; q < NQ_MAX_RANKS; ++q)
        peers.region[q] = q < P ? comm->peer[q] + kArenaHeader + arena_offset : nullptr;
    unsigned int *epoch = reinterpret_cast<unsigned int *>(comm->arena + kEpochOff);
    unsigned int *err = reinterpret_cast<unsigned int *>(comm->arena + kErrOff);
    const int e_pad = P > 1 ? (int)((e0 + ne) % E) : 0;

    if (int rc = from_cuda(cudaMemsetAsync(loc.send_cnt, 0, sizeof(int32_t) * P, st), what))
        return rc;
    // ready: this rank's earlier stream work (which read its region) is done
    if (int rc = from_cuda(launch_pdl_k(push_ready_kernel, 1, 32, st,
                                        reinterpret_cast<unsigned int *const *>(comm->arena +
                                                                                kTableOff),
                                        P, epoch),
                           what))
        return rc;
    const unsigned dblocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((cap + 7) / 8, 148 * 4));
    if (int rc = from_cuda(
            launch_pdl_k(ep_dispatch_kernel, dblocks, 256, st, x_shard, topk_idx_shard,
                         topk_scores_shard, cap, H, (int)top_k, (int)E, (int)ne, P, rank, peers, rg,
                         loc.send_cnt, loc.pos,
                         reinterpret_cast<const unsigned *>(comm->arena + kReadyOff),
                         (const unsigned *)epoch, err),
            what))
        return rc;
    if (int rc = from_cuda(
            launch_pdl_k(ep_exchange_kernel, 1, 256, st, peers, rg, P, rank, cap, (int)top_k,
                         e_pad, (const int32_t *)loc.send_cnt,
                         reinterpret_cast<unsigned int *const *>(comm->arena + kDispTableOff),
                         reinterpret_cast<const unsigned *>(comm->arena + kDispOff),
                         (const unsigned *)epoch, err),
            what))
        return rc;
    // this rank's experts over every row it received; the partial sums go
    // straight back into the token owners' regions
    nq_rows_push_t push;
    std::memset(&push, 0, sizeof(push));
    push.nranks = P;
    push.rows_per_rank = cap;
    push.dst_row0 = (int64_t)rank * cap;
    push.count = reinterpret_cast<const int32_t *>(peers.region[rank] + rg.cnt);
    for (int q = 0; q < P; ++q) push.dst[q] = reinterpret_cast<float *>(peers.region[q] + rg.back);
    char *mine = peers.region[rank];
    if (int rc = from_nq(nq_moe_switch_partial_push(
                             reinterpret_cast<const uint16_t *>(mine + rg.x), T, H, I, E, top_k,
                             reinterpret_cast<const int32_t *>(mine + rg.idx),
                             reinterpret_cast<const float *>(mine + rg.sc), e0, ne, gate_w, gate_s,
                             gate_b, up_w, up_s, up_b, down_w, down_s, down_b, bits, group_size,
                             loc.sw, loc.sw_bytes, &push, stream),
                         what))
        return rc;
    // combined: every rank's partial sums for this rank's tokens have arrived
    if (int rc = from_cuda(
            launch_pdl_1warp(st, push_finish_kernel,
                             reinterpret_cast<unsigned int *const *>(comm->arena + kCombTableOff),
                             reinterpret_cast<const unsigned int *>(comm->arena + kCombOff), P,
                             epoch, err),
            what))
        return rc;
    const int64_t n4 = cap * (H / 4);
    return from_cuda(launch_pdl_k(ep_final_kernel, (unsigned)((n4 + 255) / 256), 256, st,
                                  reinterpret_cast<const float *>(mine + rg.back),
                                  (const int32_t *)loc.pos, cap, H, P, y_shard),
                     what);
}

int nq_ep_moe_switch_fused(nq_comm_t comm, const uint16_t *x_shard, int64_t T, int64_t H,
                           int64_t I, int64_t E, int64_t top_k, const int32_t *topk_idx_shard,
                           const float *topk_scores_shard, const uint32_t *gate_w,
                           const uint16_t *gate_s, const uint16_t *gate_b, const uint32_t *up_w,
                           const uint16_t *up_s, const uint16_t *up_b, const uint32_t *down_w,
                           const uint16_t *down_s, const uint16_t *down_b, int bits,
                           int group_size, size_t arena_offset, void *workspace,
                           size_t workspace_bytes, uint16_t *y_shard, void *stream) {
    if (comm && comm->aborted)
        return fail(NQ_COMPUTE_ERROR, "nq_ep_moe_switch_fused: the communicator was aborted");
    const int rc = ep_moe_switch_fused_impl(comm, x_shard, T, H, I, E, top_k, topk_idx_shard,
                                            topk_scores_shard, gate_w, gate_s, gate_b, up_w, up_s,
                                            up_b, down_w, down_s, down_b, bits, group_size,
                                            arena_offset, workspace, workspace_bytes, y_shard,
                                            stream);
    return settle(comm, stream, rc);
}

}  // extern "C"
