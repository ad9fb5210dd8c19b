// model_loader.h -- checkpoints into device memory for the CUDA backend.
//
//   ModelLoader::find_safetensors_files   mirrors compute/src/compute/model/model_loader.cpp:17-29
//   ModelLoader::load_weights_cuda        takes the place of load_model_mlx (:33-58): every
//                                         *.safetensors file of the model directory, tensors
//                                         copied unchanged (MLX layout: packed uint32 codes,
//                                         bf16 scales/biases) into device memory
//   load_quantization_config              the "quantization" block of config.json, parsed as
//                                         compute/src/compute/model/model_config.cpp:177-193
//
// Weights keep MLX's layout, so a quantized projection is ready for
// cuda_ops::lin as soon as it is loaded; each tensor keeps its own bits (read
// back from the shapes by cuda_ops::bits), so mixed-precision checkpoints
// load as they are.
#pragma once

#include <cstdint>
#include <filesystem>
#include <memory>
#include <optional>
#include <string>
#include <vector>

#include "compute_types.h"
#include "cuda_backend.h"

namespace compute {

struct QuantizationConfig {
    int group_size = 0;
    int bits = 0;
};

// config.json's optional "quantization": {"group_size": g, "bits": b}.
// nullopt when the block is absent or null; InvalidInput when a field is
// missing or the file cannot be read or parsed.
Result<std::optional<QuantizationConfig>> load_quantization_config(
    const std::filesystem::path &model_dir);

// One tensor of a safetensors file, as its header describes it.
struct SafetensorInfo {
    std::string name;
    std::string dtype;            // "U32", "BF16", "F16", "F32", "I32", ...
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // byte range inside the data section
};

// The tensors of one file (host only: reads the 8-byte length and the JSON
// header).  InvalidInput for a malformed file.
Result<std::vector<SafetensorInfo>> read_safetensors_header(const std::filesystem::path &file,
                                                            uint64_t *data_offset = nullptr);

// Device copies of every tensor of a checkpoint, with the WeightMap views the
// models use.  Owns the device memory (freed with the object).
class DeviceWeights {
public:
    DeviceWeights() = default;
    ~DeviceWeights();
    DeviceWeights(const DeviceWeights &) = delete;
    DeviceWeights &operator=(const DeviceWeights &) = delete;
    DeviceWeights(DeviceWeights &&o) noexcept;
    DeviceWeights &operator=(DeviceWeights &&o) noexcept;

    const WeightMap &map() const { return map_; }
    size_t bytes() const { return bytes_; }

private:
    friend class ModelLoader;
    WeightMap map_;
    std::vector<void *> blocks_;
    size_t bytes_ = 0;
};

class ModelLoader {
public:
    static std::vector<std::filesystem::path> find_safetensors_files(
        const std::filesystem::path &model_dir);

    // All tensors of all *.safetensors files of model_dir, on the current
    // CUDA device (copies ordered on `stream`, complete on return).
    // InvalidInput: no directory, no files, malformed header, duplicate name,
    // dtype outside {U32, I32, BF16, F16, F32}; ComputeError: device copy.
    static Result<DeviceWeights> load_weights_cuda(const std::filesystem::path &model_dir,
                                                   void *stream);
};

}  // namespace compute
