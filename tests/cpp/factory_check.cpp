// factory_check.cpp -- the host side of the integration: the reference's own
// BackendFactory / BackendManager (compute/src/compute/core/compute_backend.cpp,
// with the CUDA case of the integration notes added) linked against libnq.so,
// which supplies CUDABackend only.  Driven by tests/test_reference_factory.py;
// prints one "key value" line per result.
#include <cstdio>

#include "compute_backend.h"
#include "cuda_backend.h"

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

int main() {
    auto cuda = BackendFactory::create(BackendType::CUDA);
    std::printf("create_cuda %s\n", cuda ? "ok" : code_name(cuda.error().code));
    if (cuda) std::printf("create_cuda_type %d\n", (*cuda)->type() == BackendType::CUDA ? 1 : 0);
    auto mlx = BackendFactory::create(BackendType::MLX);
    std::printf("create_mlx %s\n", mlx ? "ok" : code_name(mlx.error().code));
    std::printf("available %zu\n", BackendFactory::available_backends().size());
    std::printf("best_is_cuda %d\n", BackendFactory::best_available_backend() == BackendType::CUDA);
    auto &mgr = BackendManager::instance();
    auto r = mgr.initialize();
    std::printf("manager_init %s\n", r ? "ok" : code_name(r.error().code));
    ComputeBackend *def = mgr.get_default_backend();
    std::printf("manager_default %s\n",
                def ? (def->type() == BackendType::CUDA ? "cuda" : "other") : "none");
    ComputeBackend *cb = mgr.get_backend(BackendType::CUDA);
    std::printf("manager_cuda %s\n", cb ? "cuda" : "none");
    mgr.cleanup();
    std::printf("cleanup ok\n");
    return 0;
}
