// dist.cu -- libnq_dist.so: tensor- and expert-parallel sharding of the
// quantized-matmul path over NCCL (one process per GPU).  Compute goes
// through libnq's C ABI (nq.h); this file adds the communicator, the
// collectives around the compute and two small layout kernels.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <cstring>
#include <string>

#include "nq.h"
#include "nq_dist.h"

struct nq_comm_s {
    ncclComm_t nccl = nullptr;
    int rank = 0;
    int size = 1;
    int device = 0;
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

// y[m, p * cols + j] = g[p][m][j]  (rank-major all-gather result -> row-major)
__global__ void rank_major_to_rows(const uint16_t *__restrict__ g, int64_t M, int64_t cols,
                                   int P, uint16_t *__restrict__ y) {
    const int64_t total = (int64_t)P * M * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % cols;
        const int64_t m = (i / cols) % M;
        const int64_t p = i / (cols * M);
        y[m * cols * P + p * cols + j] = g[i];
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

unsigned grid_for(int64_t n) {
    const int64_t b = (n + 255) / 256;
    return (unsigned)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
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

int nq_comm_destroy(nq_comm_t comm) {
    if (!comm) return NQ_SUCCESS;
    const int rc = from_nccl(ncclCommDestroy(comm->nccl), "nq_comm_destroy");
    delete comm;
    return rc;
}

int nq_comm_abort(nq_comm_t comm) {
    if (!comm) return NQ_SUCCESS;
    const int rc = from_nccl(ncclCommAbort(comm->nccl), "nq_comm_abort");
    delete comm;
    return rc;
}

int nq_comm_rank(nq_comm_t comm) { return comm ? comm->rank : -1; }
int nq_comm_size(nq_comm_t comm) { return comm ? comm->size : -1; }

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

int nq_tp_quantized_matmul(nq_comm_t comm, const uint16_t *x, int64_t M, const uint32_t *w_shard,
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
    rank_major_to_rows<<<grid_for(M * N), 256, 0, st>>>(g, M, rows, P, y);
    return from_cuda(cudaGetLastError(), what);
}

int nq_ep_moe_switch(nq_comm_t comm, const uint16_t *x_shard, int64_t T, int64_t H, int64_t I,
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

}  // extern "C"
