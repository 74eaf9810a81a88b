// Host-side packing of the tensor-core routes' weights into the operand layout the kernels
// copy straight into shared memory (chunk-major K-major, see tc.cuh), with the per-channel
// epilogue vectors of each layer.
#pragma once

#include <cstdint>
#include <vector>

#include "kernels.h"
#include "model.h"

namespace aeisu {

struct TcHostLayer {
    size_t image = 0;                  // byte offset of the B operand image
    size_t scale = 0, bias = 0;        // float offsets of the epilogue vectors
    float out_inv = 1.f, out_deq = 1.f;
};

struct TcHostPack {
    std::vector<uint8_t> bytes;        // all B images, 128-byte aligned
    std::vector<float> floats;         // stencil, epilogue vectors
    size_t stencil = 0;
    size_t project = 0, project_bias = 0;
    TcHostLayer compress, core[4], expand;
    size_t refine = 0, tail = 0, refine_bias = 0, tail_bias = 0;
    size_t head = 0;
    float slope = 0.1f, inv_s1 = 1.f;
};

// route (TcRoute of kernels.h): kRouteE4M3, the mixed route (e4m3 compress/core/expand from a
// SPYR8 artifact's FP8 weights and scales); kRouteI8, the INT8 route (int8 codes as f16 with
// the INT8 artifact's factors, biases and exact activation scales); kRouteF16, f16 weights
// everywhere.
TcHostPack pack_tc(const HostModel& m, int route);

// Operand image of a logical [N][K] matrix: chunk c, row n at (c*N + n)*16 bytes; esize 2
// (f16 bits, 8 per chunk) or 1 (e4m3 codes, 16 per chunk).  get(n, k) returns the element bits.
template <typename Get>
std::vector<uint8_t> pack_operand(int N, int K, int esize, Get get) {
    const int epc = 16 / esize, chunks = K / epc;
    std::vector<uint8_t> img(size_t(chunks) * N * 16, 0);
    for (int c = 0; c < chunks; ++c)
        for (int n = 0; n < N; ++n)
            for (int e = 0; e < epc; ++e) {
                const uint32_t v = get(n, c * epc + e);
                uint8_t* p = &img[(size_t(c) * N + n) * 16 + e * esize];
                p[0] = uint8_t(v);
                if (esize == 2) p[1] = uint8_t(v >> 8);
            }
    return img;
}

}  // namespace aeisu
