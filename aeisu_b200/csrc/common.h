// Shared host-side definitions: status exceptions and CUDA error checks.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "../../include/aeisu.h"

namespace aeisu {

// Internal failure carrying the C-ABI status it maps to.  Entry points catch it and
// return the status; nothing crosses the C boundary as an exception.
struct Error : std::runtime_error {
    int status;
    Error(int s, const std::string& msg) : std::runtime_error(msg), status(s) {}
};

[[noreturn]] inline void fail(int status, const std::string& msg) { throw Error(status, msg); }

inline void require(bool ok, const std::string& msg, int status = AEISU_ERR_INVALID_ARG) {
    if (!ok) fail(status, msg);
}

inline void cuda_check(cudaError_t e, const char* what, const char* file, int line) {
    if (e != cudaSuccess) {
        const int status = (e == cudaErrorMemoryAllocation) ? AEISU_ERR_OOM : AEISU_ERR_CUDA;
        fail(status, std::string(what) + " failed: " + cudaGetErrorString(e) + " (" + file + ":" +
                         std::to_string(line) + ")");
    }
}

}  // namespace aeisu

#define AEISU_CUDA(call) ::aeisu::cuda_check((call), #call, __FILE__, __LINE__)
