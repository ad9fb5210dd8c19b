// compute_backend.h -- the backend lifecycle interface of the compute library,
// declared as compute/src/compute/core/compute_backend.h:1-55 declares it, so
// that libnq's CUDABackend is built against the same class layout the
// reference's callers use.  Only declarations live here: the definitions of
// BackendFactory and BackendManager belong to the host application (the
// reference's compute_backend.cpp, with the CUDA case added as the
// integration notes show); libnq.so defines CUDABackend and the cuda_ops
// helpers and nothing of the factory or the manager.
//
// This directory (iface/) is on the include path only when libnq is built on
// its own.  Inside the reference tree the reference's own core/ headers are
// found instead, and cuda_backend.h compiles against them unchanged.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "compute_types.h"

namespace compute {

class ComputeBackend {
public:
    virtual ~ComputeBackend() = default;

    virtual BackendType type() const = 0;
    virtual std::string name() const = 0;
    virtual bool is_available() const = 0;

    virtual Result<void> initialize() = 0;
    virtual void cleanup() = 0;
};

class BackendFactory {
public:
    static Result<std::unique_ptr<ComputeBackend>> create(BackendType type);
    static std::vector<BackendType> available_backends();
    static BackendType best_available_backend();
};

class BackendManager {
public:
    static BackendManager &instance();

    Result<void> initialize();
    void cleanup();

    ComputeBackend *get_backend(BackendType type);
    ComputeBackend *get_default_backend();

private:
    BackendManager() = default;
    std::vector<std::unique_ptr<ComputeBackend>> backends_;
    ComputeBackend *default_backend_ = nullptr;
    bool initialized_ = false;

    void create_available_backends();
};

}  // namespace compute
