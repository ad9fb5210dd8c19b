// cuda_backend.cpp -- CUDABackend and the cuda_ops helpers.  The factory and
// the manager stay in the host application (see cuda_backend.h).
// Lifecycle mirrors MLXBackend (compute/src/compute/backends/mlx/mlx_backend.cpp:30-50):
// initialize() selects the device (mx::set_default_device(gpu) there) and
// creates the backend's stream; cleanup() releases it (mx::clear_cache there).
#include "cuda_backend.h"

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <mutex>

#include "nq.h"

namespace compute {

namespace {

Error nq_error(int st, const std::string &what) {
    ErrorCode c = ErrorCode::UnknownError;
    switch (st) {
        case NQ_INVALID_INPUT: c = ErrorCode::InvalidInput; break;
        case NQ_INVALID_MODEL: c = ErrorCode::InvalidModel; break;
        case NQ_BACKEND_NOT_AVAILABLE: c = ErrorCode::BackendNotAvailable; break;
        case NQ_COMPUTE_ERROR: c = ErrorCode::ComputeError; break;
        default: break;
    }
    return Error{c, what + ": " + nq_last_error()};
}

uint16_t *bf16p(const DeviceTensor &t) { return static_cast<uint16_t *>(t.data); }
uint32_t *u32p(const DeviceTensor &t) { return static_cast<uint32_t *>(t.data); }

}  // namespace

// ------------------------------------------------------------ CUDABackend

CUDABackend::CUDABackend(int device) : device_(device) {}

CUDABackend::~CUDABackend() { cleanup(); }

std::string CUDABackend::name() const { return "CUDA (NVIDIA B200, sm_100a)"; }

bool CUDABackend::is_available() const {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (device_ < 0 || device_ >= n) return false;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device_) != cudaSuccess) return false;
    return p.major == 10 && p.minor == 0;  // sm_100 (B200)
}

Result<void> CUDABackend::initialize() {
    if (initialized_) return {};
    if (!is_available())
        return std::unexpected(Error{ErrorCode::BackendNotAvailable,
                                     "CUDA backend needs an sm_100 (B200) device"});
    if (cudaSetDevice(device_) != cudaSuccess)
        return std::unexpected(Error{ErrorCode::ComputeError, "cudaSetDevice failed"});
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
        return std::unexpected(Error{ErrorCode::ComputeError, "cudaStreamCreate failed"});
    stream_ = s;
    initialized_ = true;
    return {};
}

void CUDABackend::cleanup() {
    if (!initialized_) return;
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
    cudaStreamDestroy(static_cast<cudaStream_t>(stream_));
    stream_ = nullptr;
    initialized_ = false;
}

Result<void> CUDABackend::synchronize() const {
    if (!initialized_) return std::unexpected(Error{ErrorCode::ComputeError, "not initialized"});
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
    if (e != cudaSuccess)
        return std::unexpected(Error{ErrorCode::ComputeError, cudaGetErrorString(e)});
    unsigned int err = 0;
    if (nq_take_device_error(&err) != NQ_SUCCESS || err != 0)
        return std::unexpected(Error{ErrorCode::ComputeError,
                                     "kernel reported device error " + std::to_string(err)});
    return {};
}

// ----------------------------------------------------------------- ops

namespace {

// cuBLAS for the dense (unquantized) linear only, loaded on first use so that
// libnq.so itself depends on nothing but the CUDA runtime.
struct CublasApi {
    using CreateFn = cublasStatus_t (*)(cublasHandle_t *);
    using SetStreamFn = cublasStatus_t (*)(cublasHandle_t, cudaStream_t);
    using GemmExFn = cublasStatus_t (*)(cublasHandle_t, cublasOperation_t, cublasOperation_t, int,
                                        int, int, const void *, const void *, cudaDataType, int,
                                        const void *, cudaDataType, int, const void *, void *,
                                        cudaDataType, int, cublasComputeType_t, cublasGemmAlgo_t);
    CreateFn create = nullptr;
    SetStreamFn set_stream = nullptr;
    GemmExFn gemm = nullptr;
    std::mutex mu;                    // a handle's stream binding + launch
    cublasHandle_t handle[64] = {};   // one per device
};

CublasApi *cublas_api() {
    static CublasApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libcublas.so.12", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libcublas.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        api.create = reinterpret_cast<CublasApi::CreateFn>(dlsym(h, "cublasCreate_v2"));
        api.set_stream = reinterpret_cast<CublasApi::SetStreamFn>(dlsym(h, "cublasSetStream_v2"));
        api.gemm = reinterpret_cast<CublasApi::GemmExFn>(dlsym(h, "cublasGemmEx"));
    });
    return api.create && api.set_stream && api.gemm ? &api : nullptr;
}

// y[M, N] = x[M, K] . w[N, K]^T in bf16 with fp32 accumulation, the
// `mx::matmul(x, swapaxes(w, 0, 1))` of mlx_ops::lin for weights without scales
// (compute/src/compute/model/mlx_ops.h:40).
Result<void> dense_lin(const DeviceTensor &x, const std::string &key, const DeviceTensor &w,
                       DeviceTensor &y, void *stream) {
    if (w.dtype != DType::BF16 || x.dtype != DType::BF16 || y.dtype != DType::BF16)
        return std::unexpected(Error{ErrorCode::InvalidModel,
                                     key + ": an unquantized linear needs bf16 weight, input and output"});
    const int64_t K = x.dim(-1);
    const int64_t M = K ? x.numel() / K : 0;
    const int64_t N = w.dim(0);
    if (w.shape.size() != 2 || w.dim(1) != K)
        return std::unexpected(Error{ErrorCode::InvalidInput, key + ": x/W inner dimension mismatch"});
    if (y.numel() != M * N)
        return std::unexpected(Error{ErrorCode::InvalidInput, key + ": output has the wrong size"});
    if (M == 0 || N == 0) return {};
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
        return std::unexpected(Error{ErrorCode::InvalidInput, key + ": shape too large"});
    CublasApi *api = cublas_api();
    if (!api)
        return std::unexpected(Error{ErrorCode::BackendNotAvailable,
                                     key + ": an unquantized linear needs cuBLAS (libcublas.so.12)"});
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return std::unexpected(Error{ErrorCode::BackendNotAvailable, key + ": no CUDA device"});
    }
    std::lock_guard<std::mutex> lk(api->mu);
    if (!api->handle[dev] && api->create(&api->handle[dev]) != CUBLAS_STATUS_SUCCESS) {
        api->handle[dev] = nullptr;
        return std::unexpected(Error{ErrorCode::ComputeError, key + ": cublasCreate failed"});
    }
    cublasHandle_t h = api->handle[dev];
    const float alpha = 1.0f, beta = 0.0f;
    // column-major view: y^T [N, M] = (w^T)^T [N, K] . x^T [K, M]
    if (api->set_stream(h, static_cast<cudaStream_t>(stream)) != CUBLAS_STATUS_SUCCESS ||
        api->gemm(h, CUBLAS_OP_T, CUBLAS_OP_N, (int)N, (int)M, (int)K, &alpha, w.data, CUDA_R_16BF,
                  (int)K, x.data, CUDA_R_16BF, (int)K, &beta, y.data, CUDA_R_16BF, (int)N,
                  CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS)
        return std::unexpected(Error{ErrorCode::ComputeError, key + ": dense bf16 GEMM failed"});
    return {};
}

}  // namespace

namespace cuda_ops {

int bits(const DeviceTensor &w, const DeviceTensor &s, int gs) {
    return nq_bits_from_shapes(w.dim(-1), s.dim(-1), gs);
}

Result<void> lin(const DeviceTensor &x, const std::string &key, const WeightMap &wm, int gs,
                 DeviceTensor &y, void *stream) {
    auto wit = wm.find(key + ".weight");
    if (wit == wm.end())
        return std::unexpected(Error{ErrorCode::InvalidModel, "missing weight " + key + ".weight"});
    const DeviceTensor &w = wit->second;
    auto sit = wm.find(key + ".scales");
    if (sit == wm.end()) return dense_lin(x, key, w, y, stream);  // unquantized layer
    const DeviceTensor &s = sit->second;
    auto bit = wm.find(key + ".biases");
    const DeviceTensor *b = bit == wm.end() ? nullptr : &bit->second;
    if (w.dtype != DType::U32 && w.dtype != DType::I32)
        return std::unexpected(Error{ErrorCode::InvalidModel, key + ".weight: packed codes must be uint32"});
    // bf16 or fp16 scales (mlx_ops.h:33-39 passes whatever the checkpoint
    // holds); the activations and the output take the scales' dtype
    const bool f16 = s.dtype == DType::F16;
    if ((s.dtype != DType::BF16 && !f16) || (b && b->dtype != s.dtype))
        return std::unexpected(Error{ErrorCode::InvalidModel,
                                     key + ": scales and biases must both be bf16 or both fp16"});
    if (x.dtype != s.dtype || y.dtype != s.dtype)
        return std::unexpected(Error{ErrorCode::InvalidInput,
                                     key + ": x and the output must have the scales' dtype"});
    const int nb = bits(w, s, gs);
    const int64_t K = x.dim(-1);
    if (K <= 0)
        return std::unexpected(Error{ErrorCode::InvalidInput, key + ": x has an empty last dimension"});
    const int64_t M = x.numel() / K;
    const int64_t N = w.dim(0);
    if (w.dim(-1) * 32 / nb != K)
        return std::unexpected(Error{ErrorCode::InvalidInput, key + ": x/W inner dimension mismatch"});
    if (y.numel() != M * N)
        return std::unexpected(Error{ErrorCode::InvalidInput, key + ": output has the wrong size"});
    const int st =
        f16 ? nq_quantized_matmul_f16(bf16p(x), M, u32p(w), bf16p(s), b ? bf16p(*b) : nullptr, N,
                                      K, nb, gs, bf16p(y), stream)
            : nq_quantized_matmul(bf16p(x), M, u32p(w), bf16p(s), b ? bf16p(*b) : nullptr, N, K,
                                  nb, gs, bf16p(y), stream);
    if (st != NQ_SUCCESS) return std::unexpected(nq_error(st, "lin(" + key + ")"));
    return {};
}

Result<void> dequantize(const DeviceTensor &w, const DeviceTensor &scales,
                        const DeviceTensor &biases, int gs, int bits, DeviceTensor &out,
                        void *stream) {
    const int64_t rows = w.numel() / w.dim(-1);
    const int64_t K = w.dim(-1) * 32 / bits;
    if (out.numel() != rows * K)
        return std::unexpected(Error{ErrorCode::InvalidInput, "dequantize: wrong output size"});
    const int st = scales.dtype == DType::F16
                       ? nq_dequantize_f16(u32p(w), bf16p(scales), bf16p(biases), rows, K, bits,
                                           gs, bf16p(out), stream)
                       : nq_dequantize(u32p(w), bf16p(scales), bf16p(biases), rows, K, bits, gs,
                                       bf16p(out), stream);
    if (st != NQ_SUCCESS) return std::unexpected(nq_error(st, "dequantize"));
    return {};
}

Result<void> gather_qmm(const DeviceTensor &x, const DeviceTensor &w, const DeviceTensor &scales,
                        const DeviceTensor &biases, const std::optional<DeviceTensor> &lhs,
                        const DeviceTensor &rhs, int gs, int bits, DeviceTensor &out,
                        void *stream) {
    if (w.shape.size() != 3)
        return std::unexpected(Error{ErrorCode::InvalidInput, "gather_qmm: w must be [E, N, K/pack]"});
    const int64_t E = w.dim(0), N = w.dim(1), K = w.dim(2) * 32 / bits;
    const int64_t M = x.shape.size() >= 2 ? x.dim(-2) : 1;
    const int64_t xb = x.numel() / (M * K);
    const int64_t n = rhs.numel();
    if (out.numel() != n * M * N)
        return std::unexpected(Error{ErrorCode::InvalidInput, "gather_qmm: wrong output size"});
    const int st = nq_gather_qmm(bf16p(x), xb, M, lhs ? static_cast<int32_t *>(lhs->data) : nullptr,
                                 static_cast<int32_t *>(rhs.data), n, u32p(w), bf16p(scales),
                                 bf16p(biases), E, N, K, bits, gs, bf16p(out), stream);
    if (st != NQ_SUCCESS) return std::unexpected(nq_error(st, "gather_qmm"));
    return {};
}

}  // namespace cuda_ops
}  // namespace compute
