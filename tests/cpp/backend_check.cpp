// backend_check.cpp -- exercises the C++ layer of libnq the way a reference
// model would: CUDABackend's lifecycle (the MLXBackend counterpart,
// mlx_backend.cpp:30-50),
// cuda_ops::bits and cuda_ops::lin (mlx_ops.h:20-42), and the checkpoint
// loader (model_loader.cpp:17-58, model_config.cpp:177-193).  Driven by
// tests/test_cpp_backend.py; prints one "key value" line per result.
//
//   backend_check backend
//   backend_check bits
//   backend_check config <model_dir>
//   backend_check header <file.safetensors>
//   backend_check lin <model_dir> <key> <x.bin> <M> <K> <out.bin>   (needs a GPU)
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "cuda_backend.h"
#include "model_loader.h"

using namespace compute;

static const char *code_name(ErrorCode c) {
    switch (c) {
        case ErrorCode::Success: return "Success";
        case ErrorCode::InvalidInput: return "InvalidInput";
        case ErrorCode::InvalidModel: return "InvalidModel";
        case ErrorCode::BackendNotAvailable: return "BackendNotAvailable";
        case ErrorCode::ComputeError: return "ComputeError";
        default: return "UnknownError";
    }
}

int main(int argc, char **argv) {
    if (argc < 2) return 2;
    const std::string cmd = argv[1];
    if (cmd == "backend") {
        CUDABackend be(0);
        std::printf("available %d\n", be.is_available() ? 1 : 0);
        auto r = be.initialize();
        std::printf("initialize %s\n", r ? "ok" : code_name(r.error().code));
        std::printf("type_cuda %d\n", be.type() == BackendType::CUDA ? 1 : 0);
        if (r) {
            std::printf("stream %d\n", be.stream() != nullptr ? 1 : 0);
            auto s = be.synchronize();
            std::printf("synchronize %s\n", s ? "ok" : code_name(s.error().code));
            be.cleanup();
            std::printf("cleanup ok\n");
        }
        return 0;
    }
    if (cmd == "bits") {
        DeviceTensor w, s;
        const int cases[][3] = {{512, 64, 64}, {1024, 64, 64}, {96, 12, 64}, {0, 64, 64}};
        for (auto &c : cases) {
            w.shape = {8, c[0]};
            s.shape = {8, c[1]};
            std::printf("bits %d\n", cuda_ops::bits(w, s, c[2]));
        }
        return 0;
    }
    if (cmd == "config" && argc >= 3) {
        auto q = load_quantization_config(argv[2]);
        if (!q) {
            std::printf("error %s\n", code_name(q.error().code));
            return 0;
        }
        if (!*q) std::printf("quantization none\n");
        else std::printf("quantization %d %d\n", (*q)->group_size, (*q)->bits);
        return 0;
    }
    if (cmd == "header" && argc >= 3) {
        uint64_t off = 0;
        auto h = read_safetensors_header(argv[2], &off);
        if (!h) {
            std::printf("error %s\n", code_name(h.error().code));
            return 0;
        }
        std::printf("data_offset %llu\n", (unsigned long long)off);
        for (auto &t : *h) {
            std::printf("tensor %s %s", t.name.c_str(), t.dtype.c_str());
            for (auto d : t.shape) std::printf(" %lld", (long long)d);
            std::printf("\n");
        }
        return 0;
    }
    if (cmd == "lin" && argc >= 8) {
        CUDABackend be(0);
        if (auto r = be.initialize(); !r) {
            std::printf("error %s\n", code_name(r.error().code));
            return 0;
        }
        auto w = ModelLoader::load_weights_cuda(argv[2], be.stream());
        if (!w) {
            std::printf("error %s %s\n", code_name(w.error().code), w.error().message.c_str());
            return 0;
        }
        std::printf("tensors %zu bytes %zu\n", w->map().size(), w->bytes());
        const std::string key = argv[3];
        const long M = std::stol(argv[5]), K = std::stol(argv[6]);
        std::vector<uint16_t> xh(M * K);
        std::ifstream(argv[4], std::ios::binary).read(reinterpret_cast<char *>(xh.data()),
                                                      (std::streamsize)(xh.size() * 2));
        const long N = w->map().at(key + ".weight").dim(0);
        void *xd = nullptr, *yd = nullptr;
        cudaMalloc(&xd, xh.size() * 2);
        cudaMalloc(&yd, (size_t)M * N * 2);
        cudaMemcpy(xd, xh.data(), xh.size() * 2, cudaMemcpyHostToDevice);
        // activations take the scales' dtype (bf16, or fp16 for an fp16 checkpoint)
        auto sit = w->map().find(key + ".scales");
        const DType act = sit != w->map().end() && sit->second.dtype == DType::F16 ? DType::F16
                                                                                  : DType::BF16;
        DeviceTensor x{xd, {M, K}, act}, y{yd, {M, N}, act};
        const auto &qc = load_quantization_config(argv[2]);
        const int gs = qc && *qc ? (*qc)->group_size : 64;
        auto r = cuda_ops::lin(x, key, w->map(), gs, y, be.stream());
        if (!r) {
            std::printf("error %s %s\n", code_name(r.error().code), r.error().message.c_str());
            return 0;
        }
        if (auto s = be.synchronize(); !s) {
            std::printf("error %s\n", code_name(s.error().code));
            return 0;
        }
        std::vector<uint16_t> yh((size_t)M * N);
        cudaMemcpy(yh.data(), yd, yh.size() * 2, cudaMemcpyDeviceToHost);
        std::ofstream(argv[7], std::ios::binary).write(reinterpret_cast<char *>(yh.data()),
                                                       (std::streamsize)(yh.size() * 2));
        std::printf("lin ok %ld %ld\n", M, N);
        cudaFree(xd);
        cudaFree(yd);
        return 0;
    }
    return 2;
}
