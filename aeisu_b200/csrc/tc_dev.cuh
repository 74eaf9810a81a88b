// Device helpers shared by the tensor-core route kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "tc.cuh"

namespace aeisu {
namespace tcd {

using namespace tc;

constexpr int kM = 128;         // pixels per MMA tile (TMEM lanes)
constexpr int kThreads = 128;   // one thread per tile pixel / TMEM lane
constexpr int kErrTimeout = 1;  // device error code: an mbarrier wait expired

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
// LeakyReLU for a negative slope s in [0, 1] (checked when the weights are packed): then
// max(v, s*v) equals (v > 0 ? v : s*v) for every input, signed zeros and NaN included.
__device__ __forceinline__ float leaky(float v, float s) { return fmaxf(v, v * s); }

// Epilogue arithmetic on 32 accumulator columns in packed f32x2 operations (each lane rounds
// as the scalar operation would).  Per-channel vectors are read from shared memory as float2.
//   v = leaky(v * scale + bias) * post
__device__ __forceinline__ void epi_fma_leaky(float (&v)[32], const float* scale, const float* bias, float slope,
                                              float post) {
    const float2* s2 = reinterpret_cast<const float2*>(scale);
    const float2* b2 = reinterpret_cast<const float2*>(bias);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float2 a = __ffma2_rn(make_float2(v[2 * i], v[2 * i + 1]), s2[i], b2[i]);
        const float2 n = __fmul2_rn(a, make_float2(slope, slope));
        a = make_float2(fmaxf(a.x, n.x), fmaxf(a.y, n.y));
        a = __fmul2_rn(a, make_float2(post, post));
        v[2 * i] = a.x;
        v[2 * i + 1] = a.y;
    }
}
// The same with the channel vectors in a kernel-parameter struct (scale[], bias[]) at channel
// offset `off` (a constant after unrolling): the values come from the constant bank.
template <typename CP>
__device__ __forceinline__ void epi_fma_leaky_cp(float (&v)[32], const CP& cp, int off, float slope, float post) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float2 a = __ffma2_rn(make_float2(v[2 * i], v[2 * i + 1]),
                              make_float2(cp.scale[off + 2 * i], cp.scale[off + 2 * i + 1]),
                              make_float2(cp.bias[off + 2 * i], cp.bias[off + 2 * i + 1]));
        const float2 n = __fmul2_rn(a, make_float2(slope, slope));
        a = make_float2(fmaxf(a.x, n.x), fmaxf(a.y, n.y));
        a = __fmul2_rn(a, make_float2(post, post));
        v[2 * i] = a.x;
        v[2 * i + 1] = a.y;
    }
}
// INT8 route: the int8 code of an already scaled value, as the shader route's quantize_s8
// (optimized/shader/src/int8_kernels.cuh:2-4): round to nearest even, clamp to [-127, 127]
// (NaN gives 0).  Kept as a float: f16 holds every code exactly, so f16 MMAs over the codes
// accumulate the exact integer dot products (|sum| <= 576 * 127^2 < 2^24 in FP32).
__device__ __forceinline__ float s8_code(float v) { return float(max(-127, min(127, __float2int_rn(v)))); }
__device__ __forceinline__ void s8_codes32(float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = s8_code(v[i]);
}
//   v = leaky(v + bias)
__device__ __forceinline__ void epi_add_leaky(float (&v)[32], const float* bias, float slope) {
    const float2* b2 = reinterpret_cast<const float2*>(bias);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float2 a = __fadd2_rn(make_float2(v[2 * i], v[2 * i + 1]), b2[i]);
        const float2 n = __fmul2_rn(a, make_float2(slope, slope));
        v[2 * i] = fmaxf(a.x, n.x);
        v[2 * i + 1] = fmaxf(a.y, n.y);
    }
}
//   v = v + bias
__device__ __forceinline__ void epi_add(float (&v)[32], const float* bias) {
    const float2* b2 = reinterpret_cast<const float2*>(bias);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float2 a = __fadd2_rn(make_float2(v[2 * i], v[2 * i + 1]), b2[i]);
        v[2 * i] = a.x;
        v[2 * i + 1] = a.y;
    }
}

// (a*w0 + b*w1) + c*w2 without contraction, as the reference's separate tensor ops.
__device__ __forceinline__ float mix3(float a, float b, float c, float w0, float w1, float w2) {
    return __fadd_rn(__fadd_rn(__fmul_rn(a, w0), __fmul_rn(b, w1)), __fmul_rn(c, w2));
}

// The same operations on two lanes at once: packed f32x2 arithmetic rounds each lane exactly
// as the scalar instruction does, so results are bit-identical.
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {   // a - b: a + (-1)*b, one rounding
    return __ffma2_rn(b, f2(-1.f), a);
}
__device__ __forceinline__ float2 mix3x2(float2 a, float2 b, float2 c, float w0, float w1, float w2) {
    return __fadd2_rn(__fadd2_rn(__fmul2_rn(a, f2(w0)), __fmul2_rn(b, f2(w1))), __fmul2_rn(c, f2(w2)));
}

// Source pixel at padded-grid coordinate (py, px) of frame f (replicate padding by clamping).
// `lut` maps uint8 to value/255 (correctly rounded, as read_rgb's float division).
__device__ __forceinline__ float3 load_src(const SrcDesc& s, int f, int py, int px, const float* lut) {
    const int y = clampi(py - s.pad_y, 0, s.H - 1), x = clampi(px - s.pad_x, 0, s.W - 1);
    if (s.kind == 0) {
        const uint8_t* p = static_cast<const uint8_t*>(s.ptr) + ((size_t(f) * s.H + y) * s.W + x) * 3;
        return make_float3(lut[p[0]], lut[p[1]], lut[p[2]]);
    }
    const size_t plane = size_t(s.H) * s.W;
    const float* p = static_cast<const float*>(s.ptr) + size_t(f) * 3 * plane + size_t(y) * s.W + x;
    return make_float3(p[0], p[plane], p[2 * plane]);
}

// Two-step form of load_src for prefetching: fetch_src_raw issues the global loads and
// returns the raw sample (three uint8 or three float bits, one per component, so nothing
// consumes the loads yet); finish_src converts it later, once the loads have had time to land.
__device__ __forceinline__ uint3 fetch_src_raw(const SrcDesc& s, int f, int py, int px) {
    const int y = clampi(py - s.pad_y, 0, s.H - 1), x = clampi(px - s.pad_x, 0, s.W - 1);
    if (s.kind == 0) {
        const uint8_t* p = static_cast<const uint8_t*>(s.ptr) + ((size_t(f) * s.H + y) * s.W + x) * 3;
        return make_uint3(p[0], p[1], p[2]);
    }
    const size_t plane = size_t(s.H) * s.W;
    const float* p = static_cast<const float*>(s.ptr) + size_t(f) * 3 * plane + size_t(y) * s.W + x;
    return make_uint3(__float_as_uint(p[0]), __float_as_uint(p[plane]), __float_as_uint(p[2 * plane]));
}
__device__ __forceinline__ float3 finish_src(const SrcDesc& s, uint3 raw, const float* lut) {
    if (s.kind == 0) return make_float3(lut[raw.x], lut[raw.y], lut[raw.z]);
    return make_float3(__uint_as_float(raw.x), __uint_as_float(raw.y), __uint_as_float(raw.z));
}

__device__ __forceinline__ void fill_lut(float* lut) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = __fdiv_rn(float(i), 255.f);
}

// Per-CTA set-up: TMEM columns (warp 0) and `nbar` mbarriers with arrival count 1.  Then the
// kernel waits for the previous kernel of the stream (everything before this point reads only
// the model's weights).  The next kernel may launch once every CTA of this one has called
// last_item() (or exited): after its TMEM allocation, so a dependent CTA never takes TMEM
// that a CTA of this kernel still needs, and only for the last work item, so the dependents
// overlap this kernel's tail rather than occupy SMs for its whole duration.
__device__ __forceinline__ void cta_setup(uint32_t* tmem_slot, uint64_t* bars, int nbar, uint32_t ncols) {
    if (threadIdx.x < 32) tmem_alloc(tmem_slot, ncols);
    if (threadIdx.x == 0) {
        for (int i = 0; i < nbar; ++i) mbar_init(bars + i, 1);
        fence_mbar_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    grid_dep_wait();
}

// Called by a CTA when it starts its last work item (see cta_setup); `stride` is the step
// between the work items of one CTA.
__device__ __forceinline__ void last_item(long long item, long long items, long long stride) {
    if (item + stride >= items) grid_dep_launch();
}
__device__ __forceinline__ void last_item(long long item, long long items) { last_item(item, items, gridDim.x); }

__device__ __forceinline__ void cta_teardown(uint32_t tmem, uint32_t ncols) {
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (threadIdx.x < 32) tmem_free(tmem, ncols);
}

// Everyone waits (bounded) for MMA completion; returns false on expiry, uniformly.  On the
// abort path thread 0 (the issuer) gives the committed MMAs one more bounded wait so they
// land before the caller releases TMEM.
__device__ __forceinline__ bool mma_wait_all(uint64_t* bar, uint32_t& phase, int* err) {
    const bool ok = mbar_wait_bounded(bar, phase, err, kErrTimeout);
    if (__syncthreads_or(!ok)) {
        if (threadIdx.x == 0 && !ok) mbar_wait_bounded(bar, phase, err, kErrTimeout, 200000000LL);
        return false;
    }
    phase ^= 1u;
    fence_after_sync();
    return true;
}

// Copy a byte image (weights in operand layout) from global to shared memory.
__device__ __forceinline__ void copy_image(uint8_t* dst, const uint8_t* src, int bytes) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
}

// 32 f32 values -> 4 x 16 B chunks of f16.
__device__ __forceinline__ void pack_f16x32(const float (&v)[32], uint4 (&o)[4]) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
        o[c] = make_uint4(pack_half2(v[8 * c], v[8 * c + 1]), pack_half2(v[8 * c + 2], v[8 * c + 3]),
                          pack_half2(v[8 * c + 4], v[8 * c + 5]), pack_half2(v[8 * c + 6], v[8 * c + 7]));
}
// 32 f32 values -> 2 x 16 B chunks of e4m3.
__device__ __forceinline__ void pack_e4m3x32(const float (&v)[32], uint4 (&o)[2]) {
#pragma unroll
    for (int c = 0; c < 2; ++c)
        o[c] = make_uint4(e4m3x4(v[16 * c], v[16 * c + 1], v[16 * c + 2], v[16 * c + 3]),
                          e4m3x4(v[16 * c + 4], v[16 * c + 5], v[16 * c + 6], v[16 * c + 7]),
                          e4m3x4(v[16 * c + 8], v[16 * c + 9], v[16 * c + 10], v[16 * c + 11]),
                          e4m3x4(v[16 * c + 12], v[16 * c + 13], v[16 * c + 14], v[16 * c + 15]));
}

// Address of chunk c of pixel (y, x) of region r in a chunk-planar tensor [R][H][nch][W][16].
__device__ __forceinline__ uint4* cp_at(const void* base, int r, int H, int y, int nch, int c, int W, int x) {
    return reinterpret_cast<uint4*>(const_cast<uint8_t*>(static_cast<const uint8_t*>(base)) +
                                    ((((size_t)r * H + y) * nch + c) * W + x) * 16);
}

// Two 16-byte chunks to consecutive chunk positions with one 32-byte store (p 32-byte aligned):
// a warp storing pixel pairs then writes whole sectors instead of every other half.  Streaming
// (.cs): the data is read back once, by the next kernel, after far more than L2 has passed.
__device__ __forceinline__ void st_global_2x16(uint4* p, const uint4& a, const uint4& b) {
    asm volatile("st.global.cs.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 :: "l"(p), "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                 : "memory");
}

// Work decomposition of the pipelined kernels: (region, column strip of 128, band of rows).
struct StripBand {
    int r, x0, y0, y1;
};
__device__ __forceinline__ StripBand strip_band(long long item, int nstrip, int nband, int band, int H,
                                                int width = kM) {
    StripBand s;
    s.r = int(item / ((long long)nstrip * nband));
    const int b = int((item / nstrip) % nband);
    s.x0 = int(item % nstrip) * width;
    s.y0 = b * band;
    s.y1 = min(s.y0 + band, H);
    return s;
}

}  // namespace tcd
}  // namespace aeisu
