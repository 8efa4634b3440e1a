/**
 * @file common.h
 * @brief Error conventions of the voxcpm C++ API (reference include/voxcpm/common.h:42-88).
 */
#ifndef VOXCPM_COMMON_H
#define VOXCPM_COMMON_H

#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "voxcpm/tensor.h"

namespace voxcpm {

constexpr int VOXCPM_VERSION_MAJOR = 0;
constexpr int VOXCPM_VERSION_MINOR = 1;
constexpr int VOXCPM_VERSION_PATCH = 0;

#define VOXCPM_UNUSED(x) (void)(x)

// Shape violations abort, as in the reference.
#define VOXCPM_ASSERT(x)                                                             \
    do {                                                                             \
        if (!(x)) {                                                                  \
            std::fprintf(stderr, "VOXCPM_ASSERT: %s:%d: %s\n", __FILE__, __LINE__, #x); \
            std::abort();                                                            \
        }                                                                            \
    } while (0)

enum class ErrorCode {
    Success = 0,
    InvalidArgument,
    OutOfMemory,
    FileNotFound,
    InvalidFormat,
    BackendError,
    NotImplemented,
};

class VOXCPM_API Error : public std::runtime_error {
public:
    explicit Error(ErrorCode code, const std::string& message) : std::runtime_error(message), code_(code) {}
    ErrorCode code() const { return code_; }

private:
    ErrorCode code_;
};

}  // namespace voxcpm

#endif  // VOXCPM_COMMON_H
