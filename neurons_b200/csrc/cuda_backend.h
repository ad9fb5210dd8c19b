// cuda_backend.h -- the CUDA backend behind neurons' ComputeBackend interface
// and the quantized-linear helpers the models call.
//
//   ComputeBackend                    compute/src/compute/core/compute_backend.h:12-24, included
//                                     from "compute_backend.h" (the reference's own header
//                                     inside its tree; iface/ when libnq is built alone)
//   CUDABackend                       takes the place of MLXBackend
//                                     (compute/src/compute/backends/mlx/mlx_backend.h:11-25)
//   cuda_ops::bits / cuda_ops::lin    mirror mlx_ops::bits / mlx_ops::lin
//                                     (compute/src/compute/model/mlx_ops.h:20-42)
//   cuda_ops::dequantize              replaces mx::dequantize at model load
//                                     (compute/src/compute/model/llama_model.cpp:60-72)
//   cuda_ops::gather_qmm              replaces mx::gather_qmm in the MoE step
//                                     (qwen3_transformer_moe_model_mlx.cpp:69-74)
//
// The reference keeps weights as name -> mx::array; here they are device
// tensors (DeviceTensor) owned by the caller's weight map.  Every op writes
// into a caller-provided output tensor and runs asynchronously on the stream
// passed in (normally CUDABackend::stream()).
#pragma once

#include <cstdint>
#include <memory>
#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

#include "compute_backend.h"

namespace compute {

enum class DType { BF16, F32, U32, I32, F16 };

// A non-owning view of a device tensor (row-major, contiguous).
struct DeviceTensor {
    void *data = nullptr;
    std::vector<int64_t> shape;
    DType dtype = DType::BF16;

    int64_t dim(int i) const { return shape.at(i < 0 ? (int)shape.size() + i : i); }
    int64_t numel() const {
        int64_t n = 1;
        for (auto d : shape) n *= d;
        return n;
    }
};

using WeightMap = std::unordered_map<std::string, DeviceTensor>;

// The CUDA backend.  BackendFactory / BackendManager are not defined in
// libnq: the host's factory (compute_backend.cpp) gains a CUDA case that
// constructs this class.
class CUDABackend : public ComputeBackend {
public:
    explicit CUDABackend(int device = 0);
    ~CUDABackend() override;

    BackendType type() const override { return BackendType::CUDA; }
    std::string name() const override;
    bool is_available() const override;
    Result<void> initialize() override;
    void cleanup() override;

    int device() const { return device_; }
    void *stream() const { return stream_; }  // cudaStream_t
    // Waits for the stream and reports any device-side error word.
    Result<void> synchronize() const;

private:
    int device_;
    void *stream_ = nullptr;
    bool initialized_ = false;
};

namespace cuda_ops {

// mlx_ops::bits: bits = round(32 * (w.shape[-1] / s.shape[-1]) / gs), 4 if not positive.
int bits(const DeviceTensor &w, const DeviceTensor &s, int gs);

// mlx_ops::lin (compute/src/compute/model/mlx_ops.h:28-42): y = x . dequant(W)^T
// through nq_quantized_matmul when "<key>.scales" exists (biases from
// "<key>.biases"); otherwise y = x . W^T for a bf16 W, as the reference's
// mx::matmul fallback, through cuBLAS (loaded on first use; without it:
// ErrorCode::BackendNotAvailable).
Result<void> lin(const DeviceTensor &x, const std::string &key, const WeightMap &wm, int gs,
                 DeviceTensor &y, void *stream);

Result<void> dequantize(const DeviceTensor &w, const DeviceTensor &scales,
                        const DeviceTensor &biases, int gs, int bits, DeviceTensor &out,
                        void *stream);

// gather_qmm(x, w, scales, biases, lhs, rhs, transpose=true, gs, bits)
Result<void> gather_qmm(const DeviceTensor &x, const DeviceTensor &w, const DeviceTensor &scales,
                        const DeviceTensor &biases, const std::optional<DeviceTensor> &lhs,
                        const DeviceTensor &rhs, int gs, int bits, DeviceTensor &out,
                        void *stream);

}  // namespace cuda_ops
}  // namespace compute
