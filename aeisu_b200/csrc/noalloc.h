// Upscale into caller-provided device buffers using only the library's static scratch array
// (no device allocation; the first call per device and shape may fill small host-side caches
// of the array's address, kernel attributes and tensor maps); see noalloc.cu for the limits and
// the sharing rules.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace aeisu {

class Engine;

void upscale_u8_noalloc(Engine& e, const uint8_t* src, int n, int h, int w, uint8_t* dst, cudaStream_t stream);

}  // namespace aeisu
