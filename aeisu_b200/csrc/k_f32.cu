// FP32 parity route: every controller layer and the reconstruction head in FP32 on CUDA
// cores, float32 NHWC activations.  These kernels define the numerics the tensor-core
// routes are measured against; they follow aeisu/model.py:273-341 (analysis),
// 473-492 (controller) and aeisu/reconstruction.py:15-83 (head) operation for operation.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.h"
#include "kernels.h"

namespace aeisu {
namespace {

constexpr int kThreads = 128;

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Source pixel at padded-grid coordinate (py, px) of frame f, as float RGB.
__device__ __forceinline__ float3 load_src(const SrcDesc& s, int f, int py, int px) {
    const int y = clampi(py - s.pad_y, 0, s.H - 1), x = clampi(px - s.pad_x, 0, s.W - 1);
    if (s.kind == 0) {
        const uint8_t* p = static_cast<const uint8_t*>(s.ptr) + ((size_t(f) * s.H + y) * s.W + x) * 3;
        return make_float3(__fdiv_rn(float(p[0]), 255.f), __fdiv_rn(float(p[1]), 255.f),
                           __fdiv_rn(float(p[2]), 255.f));
    }
    const size_t plane = size_t(s.H) * s.W;
    const float* p = static_cast<const float*>(s.ptr) + size_t(f) * 3 * plane + size_t(y) * s.W + x;
    return make_float3(p[0], p[plane], p[2 * plane]);
}

__device__ __forceinline__ float leaky(float v, float slope) { return v > 0.f ? v : v * slope; }

// Running maximum of |activation| for calibration: `m` (>= 0, or NaN) of every active lane of
// the warp into *peak.  Non-negative floats order like their bit patterns, and a NaN (above
// +inf as bits) stays visible to the caller.
__device__ __forceinline__ void peak_max(float* peak, float m) {
    const unsigned mask = __activemask();
    const unsigned v = __reduce_max_sync(mask, __float_as_uint(m));
    if (int(threadIdx.x & 31) == __ffs(mask) - 1) atomicMax(reinterpret_cast<unsigned*>(peak), v);
}

// (a*w0 + b*w1) + c*w2 without contraction, as the reference's separate tensor ops.
__device__ __forceinline__ float mix3(float a, float b, float c, float w0, float w1, float w2) {
    return __fadd_rn(__fadd_rn(__fmul_rn(a, w0), __fmul_rn(b, w1)), __fmul_rn(c, w2));
}

// Feature analysis (model.py:273-341) for the 2x2 LR pixels of one packed pixel, pixel
// unshuffle (channel c*4 + i*2 + j), project_540 1x1 32->32 + LeakyReLU (model.py:481).
__global__ void __launch_bounds__(kThreads) k_analysis_project(SrcDesc src, RegionSet rs,
                                                               const float* __restrict__ stencil,
                                                               F32Layer proj, float* __restrict__ out,
                                                               float* feat_peak) {
    __shared__ float s_w[32 * 32];
    __shared__ float s_b[32];
    __shared__ float s_st[24];
    for (int i = threadIdx.x; i < 1024; i += blockDim.x) s_w[i] = proj.w[i];
    if (threadIdx.x < 32) s_b[threadIdx.x] = proj.b[threadIdx.x];
    if (threadIdx.x < 24) s_st[threadIdx.x] = stencil[threadIdx.x];
    __syncthreads();
    const int ph = rs.rh / 2, pw = rs.rw / 2;
    const long long total = (long long)rs.R * ph * pw;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int qx = int(idx % pw), qy = int((idx / pw) % ph), r = int(idx / ((long long)pw * ph));
    const int4 reg = rs.regions[r];
    float g[4][4];
    float3 rgb[2][2];
    for (int a = 0; a < 4; ++a)
        for (int b = 0; b < 4; ++b) {
            const int ly = clampi(2 * qy - 1 + a, 0, rs.rh - 1), lx = clampi(2 * qx - 1 + b, 0, rs.rw - 1);
            const float3 c = load_src(src, reg.x, reg.y + ly, reg.z + lx);
            g[a][b] = mix3(c.x, c.y, c.z, s_st[9], s_st[10], s_st[11]);
            if (a >= 1 && a <= 2 && b >= 1 && b <= 2) rgb[a - 1][b - 1] = c;
        }
    float f[32];
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j) {
            const int p = i * 2 + j;
            const float3 c = rgb[i][j];
            f[0 * 4 + p] = mix3(c.x, c.y, c.z, s_st[0], s_st[1], s_st[2]);
            f[1 * 4 + p] = mix3(c.x, c.y, c.z, s_st[3], s_st[4], s_st[5]);
            f[2 * 4 + p] = mix3(c.x, c.y, c.z, s_st[6], s_st[7], s_st[8]);
            f[3 * 4 + p] = g[i + 1][j + 1];
            const float ul = g[i][j], uc = g[i][j + 1], ur = g[i][j + 2];
            const float cl = g[i + 1][j], cr = g[i + 1][j + 2];
            const float dl = g[i + 2][j], dc = g[i + 2][j + 1], dr = g[i + 2][j + 2];
            const float hmid = __fsub_rn(cr, cl), vmid = __fsub_rn(dc, uc);
            f[4 * 4 + p] = mix3(__fsub_rn(ur, ul), hmid, __fsub_rn(dr, dl), s_st[12], s_st[13], s_st[14]);
            f[5 * 4 + p] = mix3(__fsub_rn(dl, ul), vmid, __fsub_rn(dr, ur), s_st[15], s_st[16], s_st[17]);
            f[6 * 4 + p] = mix3(__fsub_rn(dr, ul), vmid, hmid, s_st[18], s_st[19], s_st[20]);
            f[7 * 4 + p] = __fadd_rn(__fsub_rn(__fmul_rn(__fsub_rn(ur, dl), s_st[21]), __fmul_rn(vmid, s_st[22])),
                                     __fmul_rn(hmid, s_st[23]));
        }
    if (feat_peak) {   // calibration: the unshuffled features, the input project_540 quantises
        float m = 0.f;
        for (int k = 0; k < 32; ++k) m = fmaxf(m, fabsf(f[k]));
        peak_max(feat_peak, m);
    }
    float* o = out + idx * 32;
    for (int c = 0; c < 32; ++c) {
        float acc = 0.f;
        for (int k = 0; k < 32; ++k) acc = fmaf(s_w[c * 32 + k], f[k], acc);
        o[c] = leaky(acc + s_b[c], proj.slope);
    }
}

// compress_270: pixel_unshuffle(enc540) then 1x1 128->64 + LeakyReLU (model.py:482).
// Input channel k = c*4 + i*2 + j reads enc540 pixel (2y+i, 2x+j), channel c.
__global__ void __launch_bounds__(kThreads) k_compress(RegionSet rs, F32Layer L, const float* __restrict__ in,
                                                       float* __restrict__ out) {
    __shared__ float s_w[64 * 128];
    for (int i = threadIdx.x; i < 64 * 128; i += blockDim.x) s_w[i] = L.w[i];
    __syncthreads();
    const int lh = rs.rh / 4, lw = rs.rw / 4, pw = rs.rw / 2, ph = rs.rh / 2;
    const long long npix = (long long)lh * lw;
    const long long total = (long long)rs.R * 2 * npix;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const long long pix = idx % npix;
    const int half = int((idx / npix) % 2), r = int(idx / (2 * npix));
    const int x = int(pix % lw), y = int(pix / lw);
    float acc[32];
    for (int o = 0; o < 32; ++o) acc[o] = 0.f;
    for (int p = 0; p < 4; ++p) {
        const float* ip = in + ((size_t(r) * ph + 2 * y + (p >> 1)) * pw + 2 * x + (p & 1)) * 32;
        for (int c = 0; c < 32; ++c) {
            const float v = ip[c];
            const float* wr = s_w + (half * 32) * 128 + c * 4 + p;
            for (int o = 0; o < 32; ++o) acc[o] = fmaf(wr[o * 128], v, acc[o]);
        }
    }
    float* op = out + ((size_t(r) * lh + y) * lw + x) * 64 + half * 32;
    for (int o = 0; o < 32; ++o) op[o] = leaky(acc[o] + L.b[half * 32 + o], L.slope);
}

// 3x3 convolution, zero padding 1, `G` groups of CING inputs -> COUTG outputs, + bias,
// optional LeakyReLU.  Weights OIHW [G*COUTG][CING][3][3] staged in shared memory.
// One thread computes 32 output channels of one pixel; pixels are the fastest index so a
// warp reads each weight as one broadcast.
template <int CING, int COUTG, int G>
__global__ void __launch_bounds__(kThreads) k_conv3x3(int R, int H, int W, F32Layer L, bool act,
                                                      const float* __restrict__ in, float* __restrict__ out) {
    extern __shared__ float s_w[];
    constexpr int CIN = CING * G, COUT = COUTG * G, OB = COUT / 32;
    for (int i = threadIdx.x; i < COUT * CING * 9; i += blockDim.x) s_w[i] = L.w[i];
    __syncthreads();
    const long long npix = (long long)H * W;
    const long long total = (long long)R * OB * npix;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const long long pix = idx % npix;
    const int ob = int((idx / npix) % OB), r = int(idx / (npix * OB));
    const int x = int(pix % W), y = int(pix / W);
    const int g = (ob * 32) / COUTG;
    float acc[32];
    for (int o = 0; o < 32; ++o) acc[o] = 0.f;
    for (int ky = 0; ky < 3; ++ky) {
        const int yy = y + ky - 1;
        if (yy < 0 || yy >= H) continue;
        for (int kx = 0; kx < 3; ++kx) {
            const int xx = x + kx - 1;
            if (xx < 0 || xx >= W) continue;
            const float* ip = in + ((size_t(r) * H + yy) * W + xx) * CIN + g * CING;
            const float* wb = s_w + (size_t(ob) * 32) * CING * 9 + ky * 3 + kx;
            for (int c = 0; c < CING; ++c) {
                const float v = ip[c];
                for (int o = 0; o < 32; ++o) acc[o] = fmaf(wb[(o * CING + c) * 9], v, acc[o]);
            }
        }
    }
    float* op = out + ((size_t(r) * H + y) * W + x) * COUT + ob * 32;
    for (int o = 0; o < 32; ++o) {
        const float v = acc[o] + L.b[ob * 32 + o];
        op[o] = act ? leaky(v, L.slope) : v;
    }
}

// expand_270 1x1 64->128 + LeakyReLU, pixel_shuffle (channel c*4+i*2+j -> pixel (2y+i, 2x+j)),
// + enc540 skip (model.py:488-489).  One thread per (low pixel, phase).
__global__ void __launch_bounds__(kThreads) k_expand(RegionSet rs, F32Layer L, const float* __restrict__ low,
                                                     const float* __restrict__ enc540, float* __restrict__ dec,
                                                     float* exp_peak) {
    __shared__ float s_w[128 * 64];
    for (int i = threadIdx.x; i < 128 * 64; i += blockDim.x) s_w[i] = L.w[i];
    __syncthreads();
    const int lh = rs.rh / 4, lw = rs.rw / 4, pw = rs.rw / 2, ph = rs.rh / 2;
    const long long npix = (long long)lh * lw;
    const long long total = (long long)rs.R * 4 * npix;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const long long pix = idx % npix;
    const int p = int((idx / npix) % 4), r = int(idx / (4 * npix));
    const int x = int(pix % lw), y = int(pix / lw);
    const float* ip = low + ((size_t(r) * lh + y) * lw + x) * 64;
    float acc[32];
    for (int c = 0; c < 32; ++c) acc[c] = 0.f;
    for (int k = 0; k < 64; ++k) {
        const float v = ip[k];
        for (int c = 0; c < 32; ++c) acc[c] = fmaf(s_w[(c * 4 + p) * 64 + k], v, acc[c]);
    }
    const size_t o = ((size_t(r) * ph + 2 * y + (p >> 1)) * pw + 2 * x + (p & 1)) * 32;
    float m = 0.f;
    for (int c = 0; c < 32; ++c) {
        const float e = leaky(acc[c] + L.b[c * 4 + p], L.slope);
        m = fmaxf(m, fabsf(e));
        dec[o + c] = enc540[o + c] + e;
    }
    if (exp_peak) peak_max(exp_peak, m);   // calibration: expand_270's output before the skip add
}

// Calibration: per-channel sums of a float32 NHWC tensor [R][H][W][C] (C divides kThreads)
// into sums; with `phases`, channel c of pixel (y, x) adds to sums[c*4 + (y&1)*2 + (x&1)], the
// channel order of the pixel unshuffle that feeds the next layer, else to sums[c].
__global__ void __launch_bounds__(kThreads) k_chansum(const float* __restrict__ x, long long npix, int H, int W,
                                                      int C, bool phases, double* sums) {
    const int c = threadIdx.x % C, row = threadIdx.x / C, rows = kThreads / C;
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
    for (long long p = (long long)blockIdx.x * rows + row; p < npix; p += (long long)gridDim.x * rows) {
        const float v = x[p * C + c];
        const int k = phases ? int(((p / W) % H) & 1) * 2 + int((p % W) & 1) : 0;
        acc[k] += double(v);
    }
    for (int k = 0; k < (phases ? 4 : 1); ++k) atomicAdd(&sums[phases ? c * 4 + k : c], acc[k]);
}

// Calibration: max |x| over n floats into *peak.
__global__ void __launch_bounds__(kThreads) k_absmax(const float* __restrict__ x, long long n, float* peak) {
    float m = 0.f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(x[i]));
    peak_max(peak, m);
}

// 1x1 64->64 without activation (metadata_head, model.py:490).
__global__ void __launch_bounds__(kThreads) k_tail(long long npix, F32Layer L, const float* __restrict__ in,
                                                   float* __restrict__ out) {
    __shared__ float s_w[64 * 64];
    for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) s_w[i] = L.w[i];
    __syncthreads();
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= npix * 2) return;
    const long long pix = idx % npix;
    const int ob = int(idx / npix);
    const float* ip = in + pix * 64;
    float acc[32];
    for (int o = 0; o < 32; ++o) acc[o] = 0.f;
    for (int k = 0; k < 64; ++k) {
        const float v = ip[k];
        for (int o = 0; o < 32; ++o) acc[o] = fmaf(s_w[(ob * 32 + o) * 64 + k], v, acc[o]);
    }
    float* op = out + pix * 64 + ob * 32;
    for (int o = 0; o < 32; ++o) op[o] = acc[o] + L.b[ob * 32 + o];
}

// coefficient_clamp (reconstruction.py:15-17).
__device__ __forceinline__ float transfer(float v) {
    const float m = fabsf(v);
    if (m <= 2.f) return v;
    const float soft = fminf(__fadd_rn(2.f, __fmul_rn(0.05f, __fsub_rn(m, 2.f))), 2.5f);
    return v < 0.f ? -soft : soft;
}

// Reconstruction head (reconstruction.py:29-83): per LR pixel, clamp its 16 coefficients
// (parity-major channels, 20-26), mix base + basis into 4 phase filters of 25 taps, apply
// them to the replicate-padded 5x5 RGB neighbourhood, write the 2x2 output pixels.
__global__ void __launch_bounds__(kThreads) k_head(SrcDesc src, RegionSet rs, DstDesc dst,
                                                   const float* __restrict__ meta, const float* __restrict__ base,
                                                   const float* __restrict__ basis, int* nonfinite) {
    __shared__ float4 s_basis[25 * 16];
    __shared__ float4 s_base[25];
    for (int i = threadIdx.x; i < 400; i += blockDim.x)
        s_basis[i] = make_float4(basis[i * 4], basis[i * 4 + 1], basis[i * 4 + 2], basis[i * 4 + 3]);
    if (threadIdx.x < 25)
        s_base[threadIdx.x] = make_float4(base[threadIdx.x * 4], base[threadIdx.x * 4 + 1],
                                          base[threadIdx.x * 4 + 2], base[threadIdx.x * 4 + 3]);
    __syncthreads();
    const long long per = (long long)rs.core_h * rs.core_w;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= per * rs.R) return;
    const int r = int(idx / per);
    const int cy = int((idx % per) / rs.core_w), cx = int(idx % rs.core_w);
    const int4 core = rs.cores[r];
    const int y = core.x + cy, x = core.y + cx;
    if (y >= core.z || x >= core.w) return;
    const int4 reg = rs.regions[r];
    const int ph = rs.rh / 2, pw = rs.rw / 2;
    const int parity = ((y & 1) << 1) | (x & 1);
    const float* mp = meta + ((size_t(r) * ph + (y >> 1)) * pw + (x >> 1)) * 64 + parity * 16;
    float c[16];
    for (int k = 0; k < 16; ++k) c[k] = transfer(mp[k]);
    float acc[4][3] = {};
    for (int t = 0; t < 25; ++t) {
        const int ty = t / 5, tx = t % 5;
        const int ly = clampi(y + ty - 2, 0, rs.rh - 1), lx = clampi(x + tx - 2, 0, rs.rw - 1);
        const float3 s = load_src(src, reg.x, reg.y + ly, reg.z + lx);
        float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < 16; ++k) {
            const float4 b = s_basis[t * 16 + k];
            m.x = fmaf(c[k], b.x, m.x); m.y = fmaf(c[k], b.y, m.y);
            m.z = fmaf(c[k], b.z, m.z); m.w = fmaf(c[k], b.w, m.w);
        }
        const float4 b0 = s_base[t];
        const float w[4] = {b0.x + m.x, b0.y + m.y, b0.z + m.z, b0.w + m.w};
        for (int p = 0; p < 4; ++p) {
            acc[p][0] = fmaf(s.x, w[p], acc[p][0]);
            acc[p][1] = fmaf(s.y, w[p], acc[p][1]);
            acc[p][2] = fmaf(s.z, w[p], acc[p][2]);
        }
    }
    bool bad = false;
    for (int p = 0; p < 4; ++p) {
        const int oy = 2 * (reg.y + y - dst.pad_y) + (p >> 1), ox = 2 * (reg.z + x - dst.pad_x) + (p & 1);
        for (int ch = 0; ch < 3; ++ch) {
            const float v = acc[p][ch];
            bad |= !isfinite(v);
            if (dst.kind == 1) {
                static_cast<float*>(dst.ptr)[((size_t(reg.x) * 3 + ch) * dst.OH + oy) * dst.OW + ox] = v;
            } else {
                const float cl = fminf(fmaxf(v, 0.f), 1.f);
                static_cast<uint8_t*>(dst.ptr)[((size_t(reg.x) * dst.OH + oy) * dst.OW + ox) * 3 + ch] =
                    uint8_t(floorf(__fadd_rn(__fmul_rn(cl, 255.f), 0.5f)));
            }
        }
    }
    if (bad) atomicOr(nonfinite, 1);
}

inline unsigned blocks_for(long long n) { return unsigned((n + kThreads - 1) / kThreads); }

void set_smem(const void* fn, int bytes) {
    AEISU_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

}  // namespace

void launch_f32_controller(const SrcDesc& src, const RegionSet& rs, const float* stencil, const F32Layer* L,
                           float* enc540, float* low_a, float* low_b, float* dec540, float* refined,
                           float* meta, cudaStream_t s, int* launches, const StageMark& mark, float* peaks,
                           double* sums) {
    const long long packed = (long long)rs.R * (rs.rh / 2) * (rs.rw / 2);
    const long long low = (long long)rs.R * (rs.rh / 4) * (rs.rw / 4);
    int extra = 0;
    auto absmax = [&](const float* x, long long n, int k) {
        if (!peaks) return;
        k_absmax<<<unsigned(std::min<long long>(blocks_for(n), 4096)), kThreads, 0, s>>>(x, n, peaks + k);
        ++extra;
    };
    // input-channel sums of the FP8 layers: compress (128, unshuffle order), bottleneck 0-3 and
    // expand (64 each)
    auto chansum = [&](const float* x, long long npix, int H, int W, int C, bool phases, int off) {
        if (!sums) return;
        k_chansum<<<unsigned(std::min<long long>((npix * C + kThreads - 1) / kThreads, 1024)), kThreads, 0, s>>>(
            x, npix, H, W, C, phases, sums + off);
        ++extra;
    };
    k_analysis_project<<<blocks_for(packed), kThreads, 0, s>>>(src, rs, stencil, L[0], enc540, peaks);
    absmax(enc540, packed * 32, 1);
    chansum(enc540, packed, rs.rh / 2, rs.rw / 2, 32, true, 0);
    mark(1);
    k_compress<<<blocks_for(low * 2), kThreads, 0, s>>>(rs, L[1], enc540, low_a);
    absmax(low_a, low * 64, 2);
    chansum(low_a, low, rs.rh / 4, rs.rw / 4, 64, false, 128);
    constexpr int core_smem = 64 * 32 * 9 * 4;
    set_smem((const void*)k_conv3x3<32, 32, 2>, core_smem);
    set_smem((const void*)k_conv3x3<32, 64, 1>, core_smem);
    float* bufs[2] = {low_a, low_b};
    for (int i = 0; i < 4; ++i) {
        k_conv3x3<32, 32, 2><<<blocks_for(low * 2), kThreads, core_smem, s>>>(
            rs.R, rs.rh / 4, rs.rw / 4, L[2 + i], true, bufs[i & 1], bufs[(i + 1) & 1]);
        absmax(bufs[(i + 1) & 1], low * 64, 3 + i);
        chansum(bufs[(i + 1) & 1], low, rs.rh / 4, rs.rw / 4, 64, false, 192 + 64 * i);
    }
    mark(2);
    k_expand<<<blocks_for(low * 4), kThreads, 0, s>>>(rs, L[6], low_a, enc540, dec540, peaks ? peaks + 7 : nullptr);
    absmax(dec540, packed * 32, 8);
    mark(3);
    k_conv3x3<32, 64, 1><<<blocks_for(packed * 2), kThreads, core_smem, s>>>(
        rs.R, rs.rh / 2, rs.rw / 2, L[7], true, dec540, refined);
    absmax(refined, packed * 64, 9);
    k_tail<<<blocks_for(packed * 2), kThreads, 0, s>>>(packed, L[8], refined, meta);
    AEISU_CUDA(cudaGetLastError());
    *launches += 10 + extra;
    mark(4);
}

void launch_f32_head(const SrcDesc& src, const RegionSet& rs, const DstDesc& dst, const float* meta,
                     const float* base, const float* basis, int* nonfinite, cudaStream_t s, int* launches) {
    const long long n = (long long)rs.R * rs.core_h * rs.core_w;
    if (n == 0) return;
    k_head<<<blocks_for(n), kThreads, 0, s>>>(src, rs, dst, meta, base, basis, nonfinite);
    AEISU_CUDA(cudaGetLastError());
    *launches += 1;
}

}  // namespace aeisu
