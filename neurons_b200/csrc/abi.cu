// abi.cu -- the extern "C" entry points declared in include/nq.h: argument
// validation on the host, dispatch to the sm_100a kernels, status mapping.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "nq.h"
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

namespace {
thread_local std::string g_last_error;

// Device error word: one per device, set by kernels (bounded waits, bad
// gather indices), read and cleared by nq_take_device_error.
__device__ unsigned int g_device_error;

constexpr int kMaxDevices = 64;
unsigned int *g_err_ptr[kMaxDevices];
int g_sms[kMaxDevices];
std::mutex g_mu;

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return d;
}
}  // namespace

void set_error(const std::string &msg) { g_last_error = msg; }
const char *last_error() { return g_last_error.c_str(); }

unsigned int *device_error_word() {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_err_ptr[d]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess)
            g_err_ptr[d] = static_cast<unsigned int *>(p);
        else
            cudaGetLastError();
    }
    return g_err_ptr[d];
}

int sm_count() {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return 148;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_sms[d]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
        g_sms[d] = v > 0 ? v : 148;
    }
    return g_sms[d];
}

}  // namespace nq

using nq::set_error;

namespace {

int fail(nq_status st, const std::string &msg) {
    set_error(msg);
    return st;
}

int from_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return NQ_SUCCESS;
    // a rejected launch must not leave its status behind for the caller's next
    // CUDA call (cudaGetLastError resets it; sticky errors stay sticky anyway)
    cudaGetLastError();
    return fail(NQ_COMPUTE_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_quant(int64_t rows, int64_t K, int bits, int gs, const char *fn) {
    if (bits != 4 && bits != 8)
        return fail(NQ_INVALID_INPUT, std::string(fn) + ": bits must be 4 or 8, got " +
                                          std::to_string(bits));
    if (gs != 32 && gs != 64 && gs != 128)
        return fail(NQ_INVALID_INPUT, std::string(fn) +
                                          ": group_size must be 32, 64 or 128, got " +
                                          std::to_string(gs));
    if (rows < 0 || K <= 0)
        return fail(NQ_INVALID_INPUT, std::string(fn) + ": shapes must be positive");
    if (K % gs)
        return fail(NQ_INVALID_INPUT, std::string(fn) + ": K=" + std::to_string(K) +
                                          " is not a multiple of group_size=" + std::to_string(gs));
    return NQ_SUCCESS;
}

int need_device(const char *fn) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(NQ_BACKEND_NOT_AVAILABLE, std::string(fn) + ": no CUDA device");
    }
    return NQ_SUCCESS;
}

}  // namespace

extern "C" {

int nq_version(void) { return 1; }

const char *nq_last_error(void) { return nq::last_error(); }

int nq_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int nq_take_device_error(unsigned int *err_out) {
    if (!err_out) return fail(NQ_INVALID_INPUT, "nq_take_device_error: err_out is NULL");
    if (int rc = need_device("nq_take_device_error")) return rc;
    unsigned int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, nq::g_device_error, sizeof(v));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(nq::g_device_error, &zero, sizeof(zero));
    *err_out = v;
    return from_cuda(e, "nq_take_device_error");
}

int nq_bits_from_shapes(int64_t w_cols, int64_t s_cols, int group_size) {
    if (s_cols <= 0 || group_size <= 0) return 4;
    const double v = 32.0 * ((double)w_cols / (double)s_cols) / (double)group_size;
    const int b = (int)(v < 0 ? v - 0.5 : v + 0.5);
    return b > 0 ? b : 4;
}

int nq_quantize(const void *w, int w_dtype, int64_t rows, int64_t K, int bits, int group_size,
                int scheme, uint32_t *wq, uint16_t *scales, uint16_t *biases, void *stream) {
    if (int rc = check_quant(rows, K, bits, group_size, "nq_quantize")) return rc;
    if (w_dtype != NQ_DTYPE_F32 && w_dtype != NQ_DTYPE_BF16 && w_dtype != NQ_DTYPE_F16)
        return fail(NQ_INVALID_INPUT,
                    "nq_quantize: w_dtype must be NQ_DTYPE_F32, NQ_DTYPE_BF16 or NQ_DTYPE_F16");
    if (scheme != NQ_SCHEME_MLX_AFFINE && scheme != NQ_SCHEME_MINMAX)
        return fail(NQ_INVALID_INPUT, "nq_quantize: unknown scheme");
    if (rows == 0) return NQ_SUCCESS;
    if (!w || !wq || !scales || !biases)
        return fail(NQ_INVALID_INPUT, "nq_quantize: NULL tensor pointer");
    if (!aligned16(w) || !aligned16(wq))
        return fail(NQ_INVALID_INPUT, "nq_quantize: w and wq must be 16-byte aligned");
    if (int rc = need_device("nq_quantize")) return rc;
    return from_cuda(nq::launch_quantize(w, w_dtype, rows, K, bits, group_size, scheme, wq, scales,
                                         biases, static_cast<cudaStream_t>(stream)),
                     "nq_quantize");
}

int nq_dequantize(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases, int64_t rows,
                  int64_t K, int bits, int group_size, uint16_t *out, void *stream) {
    if (int rc = check_quant(rows, K, bits, group_size, "nq_dequantize")) return rc;
    if (rows == 0) return NQ_SUCCESS;
    if (!wq || !scales || !out) return fail(NQ_INVALID_INPUT, "nq_dequantize: NULL tensor pointer");
    if (!biases)
        return fail(NQ_INVALID_INPUT,
                    "nq_dequantize: biases must be provided for affine quantization");
    if (!aligned16(wq) || !aligned16(out))
        return fail(NQ_INVALID_INPUT, "nq_dequantize: wq and out must be 16-byte aligned");
    if (int rc = need_device("nq_dequantize")) return rc;
    return from_cuda(nq::launch_dequantize(wq, scales, biases, rows, K, bits, group_size, out,
                                           static_cast<cudaStream_t>(stream)),
                     "nq_dequantize");
}

int nq_dequantize_f16(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases,
                      int64_t rows, int64_t K, int bits, int group_size, uint16_t *out,
                      void *stream) {
    const char *what = "nq_dequantize_f16";
    if (int rc = check_quant(rows, K, bits, group_size, what)) return rc;
    if (rows == 0) return NQ_SUCCESS;
    if (!wq || !scales || !biases || !out)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL tensor pointer");
    if (!aligned16(wq) || !aligned16(out))
        return fail(NQ_INVALID_INPUT, std::string(what) + ": wq and out must be 16-byte aligned");
    if (int rc = need_device(what)) return rc;
    return from_cuda(nq::launch_dequantize(wq, scales, biases, rows, K, bits, group_size, out,
                                           static_cast<cudaStream_t>(stream), true),
                     what);
}

int nq_quantized_matmul_f16(const uint16_t *x, int64_t M, const uint32_t *wq,
                            const uint16_t *scales, const uint16_t *biases, int64_t N, int64_t K,
                            int bits, int group_size, uint16_t *y, void *stream) {
    const char *what = "nq_quantized_matmul_f16";
    if (int rc = check_quant(N, K, bits, group_size, what)) return rc;
    if (M < 0) return fail(NQ_INVALID_INPUT, std::string(what) + ": M must be >= 0");
    if (M == 0 || N == 0) return NQ_SUCCESS;
    if (!x || !wq || !scales || !biases || !y)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL tensor pointer");
    if (!aligned16(x) || !aligned16(wq))
        return fail(NQ_INVALID_INPUT, std::string(what) + ": x and wq must be 16-byte aligned");
    if (N > (1LL << 31) - 1 || M > (1LL << 31) - 1)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": shape too large");
    if (int rc = need_device(what)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (M <= 8 && bits == 4) {
        const cudaError_t e = nq::launch_rows_f16(x, (int)M, wq, scales, biases, N, K, bits,
                                                  group_size, y, st);
        if (e != cudaErrorNotSupported) return from_cuda(e, what);
    }
    nq::TcGemmArgs a;
    a.x = x; a.x_ld = K; a.M = M;
    a.w = wq; a.s = scales; a.b = biases;
    a.N = N; a.K = K; a.bits = bits; a.gs = group_size;
    a.y = y; a.y_ld = N;
    a.f16 = true;
    if (!nq::tc_gemm_supported(a))
        return fail(NQ_BACKEND_NOT_AVAILABLE,
                    std::string(what) + ": shape not served (K*bits/8 and x rows must be "
                                        "multiples of 16 bytes, and tensor maps available)");
    return from_cuda(nq::launch_tc_gemm(a, st), what);
}

// Whether the tcgen05 GEMM serves a plain M x N x K call instead of the
// mma.sync GEMVs.  The GEMM streams the weights in about the same time for
// any M up to its 64-token tile (B200, 4-bit g64: 30 us at 14336 x 4096, 14 us
// at 4096^2, 11 us at 3072^2), while a GEMV's time grows with M; measured
// crossovers:
//   * 8-bit: the GEMV only at M = 1 (4096 x 14336: 43 against 31 us at M = 2),
//     with group size 128 up to M = 8 (its GEMV stays near 28 us there);
//   * 4-bit: the row-group GEMV up to M = 8, except on weights of 32 M codes or
//     more with 8192 rows or more (14336 x 4096, M = 8: 39.8 against 30.7 us);
//     for M = 9..16 the GEMV on weights below 32 M codes (4096^2, M = 16: 11.4
//     against 14.0 us); the GEMM from M = 17 (M = 32: 105 against 31 us).
static bool tc_preferred(int64_t M, int64_t N, int64_t K, int bits, int gs) {
    if (bits != 4) return M >= (gs == 128 ? 9 : 2);
    const bool big = N * K >= ((int64_t)1 << 25);
    if (M >= 17) return true;
    if (M >= 9) return big;
    return M == 8 && big && N >= 8192;
}

// Whether a tensor-parallel fan-out (push) call takes the tcgen05 GEMM: always
// from 33 tokens (the GEMV fan-out serves at most 32), and below that wherever
// the plain call on the same shard would, so that the fused and the NCCL
// tensor-parallel paths run the same kernel and give the same bits.
static bool push_uses_tc(int64_t M, int64_t N, int64_t K, int bits, int group_size,
                         const uint16_t *x, const uint32_t *wq) {
    if (M >= 33) return true;
    if (!tc_preferred(M, N, K, bits, group_size)) return false;
    nq::TcGemmArgs a;
    a.x = x; a.x_ld = K; a.M = M;
    a.w = wq;
    a.N = N; a.K = K; a.bits = bits; a.gs = group_size;
    return nq::tc_gemm_supported(a);
}

int nq_quantized_matmul(const uint16_t *x, int64_t M, const uint32_t *wq, const uint16_t *scales,
                        const uint16_t *biases, int64_t N, int64_t K, int bits, int group_size,
                        uint16_t *y, void *stream) {
    if (int rc = check_quant(N, K, bits, group_size, "nq_quantized_matmul")) return rc;
    if (M < 0) return fail(NQ_INVALID_INPUT, "nq_quantized_matmul: M must be >= 0");
    if (M == 0 || N == 0) return NQ_SUCCESS;
    if (!x || !wq || !scales || !y)
        return fail(NQ_INVALID_INPUT, "nq_quantized_matmul: NULL tensor pointer");
    if (!biases)
        return fail(NQ_INVALID_INPUT,
                    "nq_quantized_matmul: biases must be provided for affine quantization");
    if (!aligned16(x) || !aligned16(wq))
        return fail(NQ_INVALID_INPUT, "nq_quantized_matmul: x and wq must be 16-byte aligned");
    if (N > 16 * 65535LL * 65535LL || M > (1LL << 31) - 1)
        return fail(NQ_INVALID_INPUT, "nq_quantized_matmul: shape too large");
    if (int rc = need_device("nq_quantized_matmul")) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (tc_preferred(M, N, K, bits, group_size)) {
        nq::TcGemmArgs a;
        a.x = x; a.x_ld = K; a.M = M;
        a.w = wq; a.s = scales; a.b = biases;
        a.N = N; a.K = K; a.bits = bits; a.gs = group_size;
        a.y = y; a.y_ld = N;
        if (nq::tc_gemm_supported(a))
            return from_cuda(nq::launch_tc_gemm(a, st), "nq_quantized_matmul");
    }
    nq::GemvProblems p;
    p.w = wq; p.s = scales; p.b = biases;
    p.N = N; p.K = K; p.bits = bits; p.gs = group_size;
    p.x = x; p.x_ld = K;
    p.P = 1; p.M = (int)M; p.max_m = (int)M;
    p.y = y; p.y_ld = N;
    return from_cuda(nq::launch_gemv(p, st), "nq_quantized_matmul");
}

int nq_quantized_matmul_launches(int64_t M, int64_t N, int64_t K, int bits, int group_size) {
    if (int rc = check_quant(N, K, bits, group_size, "nq_quantized_matmul_launches")) return rc;
    if (M < 0) return fail(NQ_INVALID_INPUT, "nq_quantized_matmul_launches: M must be >= 0");
    if (M == 0 || N == 0) return 0;
    if (int rc = need_device("nq_quantized_matmul_launches")) return rc;
    if (tc_preferred(M, N, K, bits, group_size)) {
        // the shape alone decides; any 16-byte aligned operands take the same path
        static const uint4 aligned_probe[1] = {};
        nq::TcGemmArgs a;
        a.x = reinterpret_cast<const uint16_t *>(aligned_probe); a.x_ld = K; a.M = M;
        a.w = reinterpret_cast<const uint32_t *>(aligned_probe);
        a.N = N; a.K = K; a.bits = bits; a.gs = group_size; a.y_ld = N;
        if (const int n = nq::tc_gemm_launches(a)) return n;
    }
    return 1;
}

}  // extern "C"

// Everything nq_quantized_matmul_push checks before it launches, in one place,
// so that a caller can validate a fused call before any other work of the
// call is enqueued.  Device-independent checks come first.
static int push_validate(const char *what, const uint16_t *x, int64_t M, const uint32_t *wq,
                         const uint16_t *scales, const uint16_t *biases, int64_t N, int64_t K,
                         int bits, int group_size, int64_t N_total, int64_t col0,
                         const nq_push_t *push) {
    if (int rc = check_quant(N, K, bits, group_size, what)) return rc;
    if (M <= 0 || N <= 0) return fail(NQ_INVALID_INPUT, std::string(what) + ": M and N must be > 0");
    if (!x || !wq || !scales || !biases || !push)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL pointer");
    if (push->nranks < 1 || push->nranks > NQ_MAX_RANKS || push->rank < 0 ||
        push->rank >= push->nranks)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": need 0 <= rank < nranks <= 8");
    if (col0 < 0 || col0 + N > N_total)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": columns outside [0, N_total)");
    if (!push->ready || !push->epoch)
        return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL flag pointer");
    for (int q = 0; q < push->nranks; ++q)
        if (!push->dst[q]) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL destination");
    if (!aligned16(x) || !aligned16(wq))
        return fail(NQ_INVALID_INPUT, std::string(what) + ": x and wq must be 16-byte aligned");
    if (push_uses_tc(M, N, K, bits, group_size, x, wq)) {
        nq::TcGemmArgs a;
        a.x = x; a.x_ld = K; a.M = M;
        a.w = wq; a.s = scales; a.b = biases;
        a.N = N; a.K = K; a.bits = bits; a.gs = group_size;
        a.y_ld = N_total;
        if ((a.x_ld * 2) % 16 || (K * bits / 8) % 16)
            return fail(NQ_INVALID_INPUT,
                        std::string(what) + ": K*bits/8 must be a multiple of 16 bytes");
        if (int rc = need_device(what)) return rc;
        if (!nq::tc_gemm_supported(a))
            return fail(NQ_INVALID_INPUT, std::string(what) + ": shape not served by the fused path");
        return NQ_SUCCESS;
    }
    nq::GemvProblems p;
    p.w = wq; p.s = scales; p.b = biases;
    p.N = N; p.K = K; p.bits = bits; p.gs = group_size;
    p.x = x; p.x_ld = K;
    if (const char *why = nq::gemv_push_unsupported(p))
        return fail(NQ_INVALID_INPUT, std::string(what) + ": " + why);
    if (int rc = need_device(what)) return rc;
    if (!nq::tensor_maps_available())
        return fail(NQ_BACKEND_NOT_AVAILABLE,
                    std::string(what) + ": the driver provides no tensor-map encoder");
    return NQ_SUCCESS;
}

extern "C" {

int nq_quantized_matmul_push_check(const uint16_t *x, int64_t M, const uint32_t *wq,
                                   const uint16_t *scales, const uint16_t *biases, int64_t N,
                                   int64_t K, int bits, int group_size, int64_t N_total,
                                   int64_t col0, const nq_push_t *push) {
    return push_validate("nq_quantized_matmul_push", x, M, wq, scales, biases, N, K, bits,
                         group_size, N_total, col0, push);
}

int nq_quantized_matmul_push(const uint16_t *x, int64_t M, const uint32_t *wq,
                             const uint16_t *scales, const uint16_t *biases, int64_t N, int64_t K,
                             int bits, int group_size, int64_t N_total, int64_t col0,
                             const nq_push_t *push, void *stream) {
    const char *what = "nq_quantized_matmul_push";
    if (int rc = push_validate(what, x, M, wq, scales, biases, N, K, bits, group_size, N_total,
                               col0, push))
        return rc;
    nq::PushDev pd;
    pd.n = push->nranks;
    pd.epoch = push->epoch;
    pd.ready = push->ready;
    const char *self = static_cast<const char *>(push->dst[push->rank]);
    for (int q = 0; q < pd.n; ++q) pd.delta[q] = static_cast<const char *>(push->dst[q]) - self;
    uint16_t *y = static_cast<uint16_t *>(push->dst[push->rank]) + col0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (push_uses_tc(M, N, K, bits, group_size, x, wq)) {
        nq::TcGemmArgs a;
        a.x = x; a.x_ld = K; a.M = M;
        a.w = wq; a.s = scales; a.b = biases;
        a.N = N; a.K = K; a.bits = bits; a.gs = group_size;
        a.y = y; a.y_ld = N_total;
        a.push = &pd;
        return from_cuda(nq::launch_tc_gemm(a, st), what);
    }
    nq::GemvProblems p;
    p.w = wq; p.s = scales; p.b = biases;
    p.N = N; p.K = K; p.bits = bits; p.gs = group_size;
    p.x = x; p.x_ld = K;
    p.P = 1; p.M = (int)M; p.max_m = (int)M;
    p.y = y; p.y_ld = N_total;
    p.push = &pd;
    return from_cuda(nq::launch_gemv(p, st), what);
}

int nq_gather_qmm(const uint16_t *x, int64_t x_batch, int64_t M, const int32_t *lhs_indices,
                  const int32_t *rhs_indices, int64_t n_idx, const uint32_t *wq,
                  const uint16_t *scales, const uint16_t *biases, int64_t E, int64_t N, int64_t K,
                  int bits, int group_size, uint16_t *y, void *stream) {
    if (int rc = check_quant(N, K, bits, group_size, "nq_gather_qmm")) return rc;
    if (M < 0 || n_idx < 0 || E <= 0 || x_batch <= 0)
        return fail(NQ_INVALID_INPUT, "nq_gather_qmm: invalid batch/expert sizes");
    if (!lhs_indices && x_batch != 1 && x_batch != n_idx)
        return fail(NQ_INVALID_INPUT,
                    "nq_gather_qmm: without lhs_indices x_batch must be 1 or equal n_idx");
    if (M == 0 || N == 0 || n_idx == 0) return NQ_SUCCESS;
    if (n_idx > 65535) return fail(NQ_INVALID_INPUT, "nq_gather_qmm: at most 65535 indices");
    if (!x || !rhs_indices || !wq || !scales || !y)
        return fail(NQ_INVALID_INPUT, "nq_gather_qmm: NULL tensor pointer");
    if (!biases)
        return fail(NQ_INVALID_INPUT,
                    "nq_gather_qmm: biases must be provided for affine quantization");
    if (!aligned16(x) || !aligned16(wq))
        return fail(NQ_INVALID_INPUT, "nq_gather_qmm: x and wq must be 16-byte aligned");
    if (int rc = need_device("nq_gather_qmm")) return rc;
    nq::GemvProblems p;
    p.w = wq; p.s = scales; p.b = biases;
    p.N = N; p.K = K; p.bits = bits; p.gs = group_size;
    p.x = x; p.x_ld = K;
    p.P = (int)n_idx; p.M = (int)M; p.max_m = (int)M;
    p.E = (int)E;
    p.expert = rhs_indices;
    p.lhs = lhs_indices;
    p.x_batch = (int)x_batch;
    p.y = y; p.y_ld = N;
    return from_cuda(nq::launch_gemv(p, static_cast<cudaStream_t>(stream)), "nq_gather_qmm");
}

int nq_moe_route(const uint16_t *logits, int64_t T, int64_t E, int64_t top_k, int32_t *topk_idx,
                 float *topk_scores, void *stream) {
    if (T < 0 || E <= 0 || E > 1024 || top_k <= 0 || top_k > 32 || top_k > E)
        return fail(NQ_INVALID_INPUT, "nq_moe_route: need 0 < top_k <= min(E, 32), E <= 1024");
    if (T == 0) return NQ_SUCCESS;
    if (!logits || !topk_idx || !topk_scores)
        return fail(NQ_INVALID_INPUT, "nq_moe_route: NULL tensor pointer");
    if (int rc = need_device("nq_moe_route")) return rc;
    return from_cuda(nq::launch_moe_route(logits, T, E, top_k, topk_idx, topk_scores,
                                          static_cast<cudaStream_t>(stream)),
                     "nq_moe_route");
}

size_t nq_moe_workspace_size(int64_t T, int64_t E, int64_t top_k, int64_t H, int64_t I) {
    if (T < 0 || E <= 0 || top_k <= 0 || H <= 0 || I <= 0) return 0;
    return nq::moe_workspace_bytes(T, E, top_k, H, I);
}

}  // extern "C"

// Shared validation and launch of nq_moe_switch / nq_moe_switch_partial: the
// weights passed hold experts [e0, e0 + ne) of E.
static int moe_switch_checked(const char *what, const uint16_t *x, int64_t T, int64_t H, int64_t I,
                              int64_t E, int64_t top_k, const int32_t *topk_idx,
                              const float *topk_scores, int64_t e0, int64_t ne,
                              const uint32_t *gate_w, const uint16_t *gate_s,
                              const uint16_t *gate_b, const uint32_t *up_w, const uint16_t *up_s,
                              const uint16_t *up_b, const uint32_t *down_w, const uint16_t *down_s,
                              const uint16_t *down_b, int bits, int group_size, void *workspace,
                              size_t workspace_bytes, uint16_t *y, float *y_partial,
                              void *stream, const nq::MoeRowsOut *rows_out = nullptr) {
    const std::string w(what);
    if (int rc = check_quant(I, H, bits, group_size, what)) return rc;
    if (int rc = check_quant(H, I, bits, group_size, what)) return rc;
    if (T < 0 || E <= 0 || E > 1024 || top_k <= 0 || top_k > 32 || top_k > E)
        return fail(NQ_INVALID_INPUT, w + ": need 0 < top_k <= min(E, 32), E <= 1024");
    if (e0 < 0 || ne <= 0 || e0 + ne > E)
        return fail(NQ_INVALID_INPUT, w + ": expert range outside [0, E)");
    if (H % 4) return fail(NQ_INVALID_INPUT, w + ": H must be a multiple of 4");
    if (T == 0) return NQ_SUCCESS;
    if (T * top_k > 65535 * 64) return fail(NQ_INVALID_INPUT, w + ": too many tokens for one call");
    if (!x || !topk_idx || !topk_scores || !gate_w || !gate_s || !gate_b || !up_w || !up_s ||
        !up_b || !down_w || !down_s || !down_b || !(y || y_partial || rows_out) || !workspace)
        return fail(NQ_INVALID_INPUT, w + ": NULL pointer");
    const size_t need = nq::moe_partial_workspace_bytes(T, E, ne, top_k, H, I);
    if (workspace_bytes < need)
        return fail(NQ_INVALID_INPUT,
                    w + ": workspace too small: need " + std::to_string(need) + " bytes");
    if (!aligned16(x) || !aligned16(gate_w) || !aligned16(up_w) || !aligned16(down_w) ||
        !aligned16(workspace) || !aligned16(y_partial))
        return fail(NQ_INVALID_INPUT, w + ": tensors must be 16-byte aligned");
    if (int rc = need_device(what)) return rc;
    return from_cuda(nq::launch_moe_switch(x, T, H, I, E, top_k, topk_idx, topk_scores, e0, ne,
                                           gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s,
                                           down_b, bits, group_size, workspace, y, y_partial,
                                           static_cast<cudaStream_t>(stream), rows_out),
                     what);
}

extern "C" {

int nq_moe_switch(const uint16_t *x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t top_k,
                  const int32_t *topk_idx, const float *topk_scores, const uint32_t *gate_w,
                  const uint16_t *gate_s, const uint16_t *gate_b, const uint32_t *up_w,
                  const uint16_t *up_s, const uint16_t *up_b, const uint32_t *down_w,
                  const uint16_t *down_s, const uint16_t *down_b, int bits, int group_size,
                  void *workspace, size_t workspace_bytes, uint16_t *y, void *stream) {
    if (!y && T > 0) return fail(NQ_INVALID_INPUT, "nq_moe_switch: NULL pointer");
    return moe_switch_checked("nq_moe_switch", x, T, H, I, E, top_k, topk_idx, topk_scores, 0, E,
                              gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b,
                              bits, group_size, workspace, workspace_bytes, y, nullptr, stream);
}

size_t nq_moe_partial_workspace_size(int64_t T, int64_t E, int64_t ne, int64_t top_k, int64_t H,
                                     int64_t I) {
    if (T < 0 || E <= 0 || ne <= 0 || ne > E || top_k <= 0 || H <= 0 || I <= 0) return 0;
    return nq::moe_partial_workspace_bytes(T, E, ne, top_k, H, I);
}

int nq_moe_switch_partial(const uint16_t *x, int64_t T, int64_t H, int64_t I, int64_t E,
                          int64_t top_k, const int32_t *topk_idx, const float *topk_scores,
                          int64_t e0, int64_t ne, const uint32_t *gate_w, const uint16_t *gate_s,
                          const uint16_t *gate_b, const uint32_t *up_w, const uint16_t *up_s,
                          const uint16_t *up_b, const uint32_t *down_w, const uint16_t *down_s,
                          const uint16_t *down_b, int bits, int group_size, void *workspace,
                          size_t workspace_bytes, float *y_partial, void *stream) {
    if (!y_partial && T > 0) return fail(NQ_INVALID_INPUT, "nq_moe_switch_partial: NULL pointer");
    return moe_switch_checked("nq_moe_switch_partial", x, T, H, I, E, top_k, topk_idx, topk_scores,
                              e0, ne, gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s,
                              down_b, bits, group_size, workspace, workspace_bytes, nullptr,
                              y_partial, stream);
}

int nq_moe_switch_partial_push(const uint16_t *x, int64_t T, int64_t H, int64_t I, int64_t E,
                               int64_t top_k, const int32_t *topk_idx, const float *topk_scores,
                               int64_t e0, int64_t ne, const uint32_t *gate_w,
                               const uint16_t *gate_s, const uint16_t *gate_b, const uint32_t *up_w,
                               const uint16_t *up_s, const uint16_t *up_b, const uint32_t *down_w,
                               const uint16_t *down_s, const uint16_t *down_b, int bits,
                               int group_size, void *workspace, size_t workspace_bytes,
                               const nq_rows_push_t *push, void *stream) {
    const char *what = "nq_moe_switch_partial_push";
    if (!push) return fail(NQ_INVALID_INPUT, std::string(what) + ": NULL push");
    if (push->nranks < 1 || push->nranks > NQ_MAX_RANKS || push->rows_per_rank <= 0 ||
        push->rows_per_rank * push->nranks != T || push->dst_row0 < 0 || !push->count)
        return fail(NQ_INVALID_INPUT,
                    std::string(what) + ": need 1 <= nranks <= 8 regions of rows_per_rank rows "
                                        "covering the T tokens, and counts");
    nq::MoeRowsOut ro;
    ro.n = push->nranks;
    ro.per = push->rows_per_rank;
    ro.row0 = push->dst_row0;
    ro.count = push->count;
    for (int q = 0; q < push->nranks; ++q) {
        if (!push->dst[q] || !aligned16(push->dst[q]))
            return fail(NQ_INVALID_INPUT,
                        std::string(what) + ": every destination must be 16-byte aligned");
        ro.dst[q] = push->dst[q];
    }
    return moe_switch_checked(what, x, T, H, I, E, top_k, topk_idx, topk_scores, e0, ne, gate_w,
                              gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b, bits,
                              group_size, workspace, workspace_bytes, nullptr, nullptr, stream,
                              &ro);
}

}  // extern "C"
