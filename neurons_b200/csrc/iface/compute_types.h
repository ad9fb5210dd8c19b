// compute_types.h -- error and backend types of the compute library, kept
// interface-compatible with compute/src/compute/core/compute_types.h:9-32 so
// that code written against the reference's Result<T>/ErrorCode compiles
// unchanged; BackendType gains the CUDA enumerator, placed between MLX and
// Auto (the reference's header takes the same one-line edit when libnq is
// linked into it).  Used only when libnq is built on its own.
#pragma once

#include <expected>
#include <string>

namespace compute {

enum class ErrorCode {
    Success,
    InvalidInput,
    InvalidModel,
    BackendNotAvailable,
    ComputeError,
    UnknownError
};

struct Error {
    ErrorCode code;
    std::string message;

    Error(ErrorCode c, std::string msg) : code(c), message(std::move(msg)) {}
};

template <typename T>
using Result = std::expected<T, Error>;

enum class BackendType {
    MLX,   // Apple MLX framework (not built here)
    CUDA,  // NVIDIA B200 (sm_100a) kernels of libnq
    Auto   // let the factory choose
};

class ComputeBackend;

}  // namespace compute
