// Tensor-core routes (FP16 and mixed FP8-E4M3/FP16) on sm_100a: every controller layer is a
// tcgen05 implicit GEMM with M = 128 output pixels of one row, N = output channels, K =
// taps x input channels; the accumulator lives in TMEM and the epilogue (scale, bias,
// LeakyReLU, requantisation, pixel (un)shuffle, skip add, coefficient clamp) runs on the
// TMEM -> register path before one store.  The reconstruction head mixes its per-pixel
// filters on the tensor core too ([128 px x 16 coeffs] x [16 x 100 taps*phases]).
//
// Activations in HBM use a chunk-planar layout: tensor[r][y][chunk][x][16 bytes], one
// 16-byte chunk = 8 f16 or 16 e4m3 channels.  A row segment of one chunk is contiguous,
// so a warp loads/stores 512 B per instruction, and a TMA box of one row window lands in
// shared memory as exactly the K-major no-swizzle operand layout of tc.cuh.
//
// The 3x3 layers and the head are pipelined per CTA over a column strip of 128 pixels and a
// band of rows: input rows stream through a ring of shared-memory slots (TMA, zero-filled
// outside the grid = the convolution's zero padding), each row is loaded once per strip,
// the MMAs of row y+1 run while the epilogue of row y drains the other TMEM buffer.
//
// Numerics follow the reference's mixed route (SrcPyrCudaRuntime.cu:4131-4873):
//   project  f16 x f16, +bias, LeakyReLU -> f16 skip                 (K1, 2360-2584)
//   compress e4m3(skip * 1/s1) x w8, acc*(s1*ws)+bias8, act, *1/s2     (K4, Compress.cuh:94-236)
//   core i   acc*(s[i+2]*ws)+bias8, act, *1/s[i+3] -> e4m3             (K5, Conv.cuh:414-632)
//   expand   acc*(s6*ws)+bias8, act, e4m3(*1/s7)*s7 + skip -> f16      (K8, Expand.cuh:232-305)
//   refine   f16, +bias, act -> f16; tail f16 + f16(bias) -> coefficients (K11, Refine.cuh:334-557)
//   head     clamp transfer, base + basis mix, 5x5 RGB apply          (K15, AdaptiveReconstruction.cuh:288-417)
// The FP16 route uses the same kernels with f16 operands everywhere and plain biases.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "common.h"
#include "kernels.h"
#include "tc_dev.cuh"
#include "tmap.h"

namespace aeisu {
namespace {

using namespace tc;
using namespace tcd;

// ---- stage 1: feature analysis + unshuffle + project_540 ------------------------------------
// Work item: a strip of 128 packed pixels and a band of packed rows.  The LR source rows the
// strip needs (2qy-1 .. 2qy+2, 258 columns) slide through a 6-row ring in shared memory as
// (r, g, b, luma) float4, so each source pixel is read and mixed once per strip (a row qy reads
// four rows while the two the previous step loaded are stored: six in all, so five CTAs fit
// an SM's shared memory).  Per packed
// row qy: the raw loads of rows 2qy+5, 2qy+6 are issued, the features of row qy are computed
// into the A operand, the rows loaded during the previous step enter the ring, one barrier,
// then the MMA of row qy runs while the epilogue of row qy-1 drains the other TMEM buffer.
// A = 32 features (f16) of the strip's packed pixels; B = project weights [32][32].
// Writes enc540 (f16, 4 chunks, packed grid: the skip input of expand) and the compress
// input at low resolution, unshuffled with K order phase*32 + c (f16: 16 chunks, e4m3: 8).
constexpr int kProjRing = 6;
constexpr int kProjTW = 2 * kM + 2;   // 258 LR columns per strip

template <bool FP8, bool I8, bool SRC_U8>
__global__ void __launch_bounds__(kThreads) k_tc_project(SrcDesc src, RegionSet rs, const ProjParams pp,
                                                         const uint8_t* __restrict__ wimg,
                                                         float slope, float inv_s1, void* __restrict__ enc540,
                                                         void* __restrict__ encu, int band, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* sA = smem;                                        // [2][4 chunks][128][16 B]
    uint8_t* sB = smem + 2 * 4 * kM * 16;                      // [4][32][16 B]
    float4 (*s_src)[kProjTW] = reinterpret_cast<float4 (*)[kProjTW]>(sB + 4 * 32 * 16);
    __shared__ float s_lut[256];
    __shared__ uint32_t s_tmem;
    __shared__ alignas(8) uint64_t s_bar[2];
    copy_image(sB, wimg, 4 * 32 * 16);
    if (SRC_U8) fill_lut(s_lut);
    const float* s_st = pp.st;   // kernel parameters: the constant bank
    fence_async_smem();
    cta_setup(&s_tmem, s_bar, 2, 64);
    const uint32_t tmem = s_tmem;
    uint32_t phase = 0, pend = 0;   // bit b: parity of buffer b's next commit / a commit not yet waited for
    const int ph = rs.rh / 2, pw = rs.rw / 2, lh = rs.rh / 4, lw = rs.rw / 4;
    const int nstrip = (pw + kM - 1) / kM, nband = (ph + band - 1) / band;
    const long long items = (long long)rs.R * nstrip * nband;
    const int t = threadIdx.x, warp = t >> 5;
    const uint32_t a0 = smem_addr(sA), b0 = smem_addr(sB);
    constexpr int PER = (kProjTW + kThreads - 1) / kThreads;   // staged columns per thread (3)
    // Column j of this thread: t and t + 128, and the last two threads also stage the two
    // columns beyond 256; warp 1 issues the MMAs.  The extra work sits in different warps
    // from the first, so no warp arrives late at the row barrier carrying both.
    constexpr int kLast = kProjTW - (PER - 1) * kThreads;     // columns of the last pass (2)
    auto col_of = [&](int j) { return j < PER - 1 ? t + j * kThreads : t - (kThreads - kLast) + (PER - 1) * kThreads; };
    auto stages = [&](int j) { return j < PER - 1 || t >= kThreads - kLast; };
    const int issuer = 32;
    bool ok = true;
    for (long long item = blockIdx.x; item < items && ok; item += gridDim.x) {
        last_item(item, items);
        const StripBand sb = strip_band(item, nstrip, nband, band, ph);
        const int4 reg = rs.regions[sb.r];
        const int base_row = 2 * sb.y0 - 1;
        auto slot = [&](int row) { return (row - base_row) % kProjRing; };   // row >= base_row
        // source columns this thread stages, clamped once per item
        int sx[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j)
            sx[j] = clampi(reg.z + clampi(2 * sb.x0 - 1 + col_of(j), 0, rs.rw - 1) - src.pad_x, 0, src.W - 1);
        auto raw_at = [&](int row, int j) -> uint3 {
            const int sy = clampi(reg.y + clampi(row, 0, rs.rh - 1) - src.pad_y, 0, src.H - 1);
            if (SRC_U8) {
                const uint8_t* p = static_cast<const uint8_t*>(src.ptr) + ((size_t(reg.x) * src.H + sy) * src.W + sx[j]) * 3;
                return make_uint3(p[0], p[1], p[2]);
            }
            const size_t plane = size_t(src.H) * src.W;
            const float* p = static_cast<const float*>(src.ptr) + size_t(reg.x) * 3 * plane + size_t(sy) * src.W + sx[j];
            return make_uint3(__float_as_uint(p[0]), __float_as_uint(p[plane]), __float_as_uint(p[2 * plane]));
        };
        auto put = [&](int row, int j, uint3 raw) {
            const float3 v = SRC_U8 ? make_float3(s_lut[raw.x], s_lut[raw.y], s_lut[raw.z])
                                    : make_float3(__uint_as_float(raw.x), __uint_as_float(raw.y), __uint_as_float(raw.z));
            s_src[slot(row)][col_of(j)] = make_float4(v.x, v.y, v.z, mix3(v.x, v.y, v.z, s_st[9], s_st[10], s_st[11]));
        };
        auto fetch2 = [&](int row, uint3 (&pre)[2][PER]) {   // raw loads of rows row, row+1
#pragma unroll
            for (int k = 0; k < 2; ++k)
#pragma unroll
                for (int j = 0; j < PER; ++j)
                    if (stages(j)) pre[k][j] = raw_at(row + k, j);
        };
        auto put2 = [&](int row, const uint3 (&pre)[2][PER]) {
#pragma unroll
            for (int k = 0; k < 2; ++k)
#pragma unroll
                for (int j = 0; j < PER; ++j)
                    if (stages(j)) put(row + k, j, pre[k][j]);
        };
        // epilogue of packed row qy from TMEM buffer b: enc540 and the compress input
        auto epilogue = [&](int qy, int b) {
            bool good = mbar_wait_bounded(&s_bar[b], (phase >> b) & 1u, err, kErrTimeout);
            if (good) {
                phase ^= 1u << b;
                pend &= ~(1u << b);
            }
            fence_after_sync();
            const int qx = sb.x0 + t;
            float v[32];
            tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + b * 32, v);
#pragma unroll
#pragma unroll
            for (int i = 0; i < 16; ++i) {   // v = leaky(v + bias), as epi_add_leaky
                const float2 a = __fadd2_rn(make_float2(v[2 * i], v[2 * i + 1]), make_float2(pp.bias[2 * i], pp.bias[2 * i + 1]));
                const float2 n = __fmul2_rn(a, make_float2(slope, slope));
                v[2 * i] = fmaxf(a.x, n.x);
                v[2 * i + 1] = fmaxf(a.y, n.y);
            }
            uint4 o[4];
            pack_f16x32(v, o);
            if (qx < pw && good) {
#pragma unroll
                for (int c = 0; c < 4; ++c) *cp_at(enc540, sb.r, ph, qy, 4, c, pw, qx) = o[c];
                const int p = (qy & 1) * 2 + (qx & 1);
                if (FP8) {
                    // compress input: e4m3(f16 skip value * 1/s1), as K4's staging
                    float q[32];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const __half2* h2 = reinterpret_cast<const __half2*>(&o[c]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 w = __fmul2_rn(__half22float2(h2[e]), f2(inv_s1));
                            q[8 * c + 2 * e] = w.x;
                            q[8 * c + 2 * e + 1] = w.y;
                        }
                    }
                    uint4 o8[2];
                    pack_e4m3x32(q, o8);
#pragma unroll
                    for (int c = 0; c < 2; ++c) *cp_at(encu, sb.r, lh, qy >> 1, 8, p * 2 + c, lw, qx >> 1) = o8[c];
                } else if (I8) {
                    // compress input: int8 codes of (f16 skip value * 1/s1), held as f16
                    // (int8_kernels.cuh:26: quantize_s8(skip, inverse_in))
                    float q[32];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const __half2* h2 = reinterpret_cast<const __half2*>(&o[c]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 w = __fmul2_rn(__half22float2(h2[e]), f2(inv_s1));
                            q[8 * c + 2 * e] = s8_code(w.x);
                            q[8 * c + 2 * e + 1] = s8_code(w.y);
                        }
                    }
                    uint4 o16[4];
                    pack_f16x32(q, o16);
#pragma unroll
                    for (int c = 0; c < 4; ++c) *cp_at(encu, sb.r, lh, qy >> 1, 16, p * 4 + c, lw, qx >> 1) = o16[c];
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c) *cp_at(encu, sb.r, lh, qy >> 1, 16, p * 4 + c, lw, qx >> 1) = o[c];
                }
            }
            return good;
        };
        // prologue: rows 2y0-1 .. 2y0+2 converted now, rows 2y0+3, 2y0+4 in flight
        for (int row = base_row; row <= 2 * sb.y0 + 2; ++row)
#pragma unroll
            for (int j = 0; j < PER; ++j)
                if (stages(j)) put(row, j, raw_at(row, j));
        uint3 pre_cur[2][PER];
        if (sb.y0 + 1 < sb.y1) fetch2(2 * sb.y0 + 3, pre_cur);
        __syncthreads();
        for (int qy = sb.y0; qy < sb.y1; ++qy) {
            const int b = (qy - sb.y0) & 1;
            uint3 pre_next[2][PER];
            if (qy + 2 < sb.y1) fetch2(2 * qy + 5, pre_next);
            // features of packed pixel (qy, qx), exactly as the FP32 route
            const int qx = sb.x0 + t, lc = 2 * (min(qx, pw - 1) - sb.x0);   // strip column of LR 2qx-1
            float g[4][4];
            float3 rgb[2][2];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 v = s_src[slot(2 * qy - 1 + a)][lc + c];
                    g[a][c] = v.w;
                    if (a >= 1 && a <= 2 && c >= 1 && c <= 2) rgb[a - 1][c - 1] = make_float3(v.x, v.y, v.z);
                }
            // the two LR pixels of row i (j = 0, 1) as the two lanes of packed f32x2 operations
            float f[32];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float2 R = make_float2(rgb[i][0].x, rgb[i][1].x), G = make_float2(rgb[i][0].y, rgb[i][1].y),
                             B = make_float2(rgb[i][0].z, rgb[i][1].z);
                auto gp = [&](int a, int c) { return make_float2(g[a][c], g[a][c + 1]); };   // columns c, c+1
                const float2 ul = gp(i, 0), uc = gp(i, 1), ur = gp(i, 2);
                const float2 cl = gp(i + 1, 0), cr = gp(i + 1, 2);
                const float2 dl = gp(i + 2, 0), dc = gp(i + 2, 1), dr = gp(i + 2, 2);
                const float2 hmid = sub2(cr, cl), vmid = sub2(dc, uc);
                float2 v[8];
                v[0] = mix3x2(R, G, B, s_st[0], s_st[1], s_st[2]);
                v[1] = mix3x2(R, G, B, s_st[3], s_st[4], s_st[5]);
                v[2] = mix3x2(R, G, B, s_st[6], s_st[7], s_st[8]);
                v[3] = gp(i + 1, 1);
                v[4] = mix3x2(sub2(ur, ul), hmid, sub2(dr, dl), s_st[12], s_st[13], s_st[14]);
                v[5] = mix3x2(sub2(dl, ul), vmid, sub2(dr, ur), s_st[15], s_st[16], s_st[17]);
                v[6] = mix3x2(sub2(dr, ul), vmid, hmid, s_st[18], s_st[19], s_st[20]);
                v[7] = __fadd2_rn(sub2(__fmul2_rn(sub2(ur, dl), f2(s_st[21])), __fmul2_rn(vmid, f2(s_st[22]))),
                                  __fmul2_rn(hmid, f2(s_st[23])));
#pragma unroll
                for (int k = 0; k < 8; ++k) {   // feature k of LR pixel p = 2i + j is channel 4k + p
                    f[4 * k + 2 * i] = v[k].x;
                    f[4 * k + 2 * i + 1] = v[k].y;
                }
            }
            uint4 fa[4];
            pack_f16x32(f, fa);
            uint8_t* a_b = sA + b * 4 * kM * 16;
#pragma unroll
            for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(a_b + (c * kM + t) * 16) = fa[c];
            // rows 2qy+3, 2qy+4 (loaded during the previous step) enter the ring for row qy+1
            if (qy + 1 < sb.y1) put2(2 * qy + 3, pre_cur);
            fence_async_smem();
            fence_before_sync();
            if (__syncthreads_or(!ok)) { ok = false; break; }   // also spreads an epilogue failure
            if (t == issuer) {
                fence_after_sync();
                constexpr uint32_t idesc = idesc_m128(32);
#pragma unroll
                for (int k = 0; k < 2; ++k)
                    mma_f16(tmem + b * 32, sdesc(a0 + b * 4 * kM * 16 + k * 2 * kM * 16, kM * 16, 128),
                            sdesc(b0 + k * 2 * 32 * 16, 32 * 16, 128), idesc, k);
                commit(&s_bar[b]);
                pend |= 1u << b;
            }
            if (qy > sb.y0 && !epilogue(qy - 1, b ^ 1)) ok = false;
#pragma unroll
            for (int k = 0; k < 2; ++k)
#pragma unroll
                for (int j = 0; j < PER; ++j) pre_cur[k][j] = pre_next[k][j];
        }
        if (ok && sb.y1 > sb.y0 && !epilogue(sb.y1 - 1, (sb.y1 - 1 - sb.y0) & 1)) ok = false;
        if (__syncthreads_or(!ok)) ok = false;
    }
    if (!ok && t == issuer)   // abort path: let committed MMAs land before TMEM is freed
        for (int b = 0; b < 2; ++b)
            if (pend & (1u << b)) mbar_wait_bounded(&s_bar[b], (phase >> b) & 1u, err, kErrTimeout, 200000000LL);
    cta_teardown(tmem, 64);
}

// ---- 1x1 convolutions at low resolution --------------------------------------------------------
// compress_270 (K = 128, N = 64) and expand_270 (K = 64, N = 128 in phase-major order).
// FP8: A/B e4m3 (16 per chunk); else f16 (8 per chunk).
template <bool FP8, bool I8 = false>
__global__ void __launch_bounds__(kThreads) k_tc_compress(RegionSet rs, const uint8_t* __restrict__ wimg, EpiParams ep,
                                                          const ChannelParams<64> cp, const void* __restrict__ encu,
                                                          void* __restrict__ out, int* err) {
    constexpr int KCH = FP8 ? 8 : 16;   // chunks of K = 128
    constexpr int OCH = FP8 ? 4 : 8;    // chunks of the 64 outputs
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* sA = smem;                        // KCH x 128 x 16
    uint8_t* sB = smem + KCH * kM * 16;        // KCH x 64 x 16
    __shared__ uint32_t s_tmem;
    __shared__ alignas(8) uint64_t s_bar;
    copy_image(sB, wimg, KCH * 64 * 16);
    fence_async_smem();
    cta_setup(&s_tmem, &s_bar, 1, 64);
    const uint32_t tmem = s_tmem;
    uint32_t phase = 0;
    const int lh = rs.rh / 4, lw = rs.rw / 4;
    const int nseg = (lw + kM - 1) / kM;
    const long long ntiles = (long long)rs.R * lh * nseg;
    const int t = threadIdx.x, warp = t >> 5;
    const uint32_t a0 = smem_addr(sA), b0 = smem_addr(sB);
    // A operand of a tile: this thread's pixel in every K chunk; the next tile's is loaded into
    // registers while the current tile's MMA and epilogue run
    uint4 pre[KCH];
    auto fetch = [&](long long tile) {
        const int seg = int(tile % nseg), y = int((tile / nseg) % lh), r = int(tile / ((long long)nseg * lh));
        const int xc = min(seg * kM + t, lw - 1);
#pragma unroll
        for (int c = 0; c < KCH; ++c) pre[c] = *cp_at(encu, r, lh, y, KCH, c, lw, xc);
    };
    if (blockIdx.x < ntiles) fetch(blockIdx.x);
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        last_item(tile, ntiles);
        const int seg = int(tile % nseg), y = int((tile / nseg) % lh), r = int(tile / ((long long)nseg * lh));
        const int x = seg * kM + t;
#pragma unroll
        for (int c = 0; c < KCH; ++c) *reinterpret_cast<uint4*>(sA + (c * kM + t) * 16) = pre[c];
        fence_async_smem();
        __syncthreads();
        if (t == 0) {
            fence_after_sync();
            constexpr uint32_t idesc = idesc_m128(64);
#pragma unroll
            for (int k = 0; k < KCH / 2; ++k) {
                const uint64_t a = sdesc(a0 + k * 2 * kM * 16, kM * 16, 128), b = sdesc(b0 + k * 2 * 64 * 16, 64 * 16, 128);
                if (FP8) mma_e4m3(tmem, a, b, idesc, k); else mma_f16(tmem, a, b, idesc, k);
            }
            commit(&s_bar);
        }
        if (tile + gridDim.x < ntiles) fetch(tile + gridDim.x);
        if (!mma_wait_all(&s_bar, phase, err)) break;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float v[32];
            tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + h * 32, v);
#pragma unroll
            epi_fma_leaky_cp(v, cp, h * 32, ep.slope, (FP8 || I8) ? ep.out_inv : 1.f);
            if (I8) s8_codes32(v);
            if (x < lw) {
                if (FP8) {
                    uint4 o[2];
                    pack_e4m3x32(v, o);
                    for (int c = 0; c < 2; ++c) *cp_at(out, r, lh, y, OCH, h * 2 + c, lw, x) = o[c];
                } else {
                    uint4 o[4];
                    pack_f16x32(v, o);
                    for (int c = 0; c < 4; ++c) *cp_at(out, r, lh, y, OCH, h * 4 + c, lw, x) = o[c];
                }
            }
        }
        fence_before_sync();
        __syncthreads();
    }
    cta_teardown(tmem, 64);
}

// expand_270 + LeakyReLU + pixel_shuffle + enc540 skip -> dec540 (f16, packed grid).
// Output channel order of B is phase-major (n = phase*32 + c), so TMEM columns
// [32p, 32p+32) are the 32 channels of output pixel (2y + p/2, 2x + p%2).
template <bool FP8, bool I8 = false>
__global__ void __launch_bounds__(kThreads, 4) k_tc_expand(RegionSet rs, const uint8_t* __restrict__ wimg, EpiParams ep,
                                                        const ChannelParams<128> cp, const void* __restrict__ low,
                                                        const void* __restrict__ enc540, void* __restrict__ dec, int* err) {
    constexpr int KCH = FP8 ? 4 : 8;   // chunks of K = 64
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* sA = smem;                        // KCH x 128 x 16
    uint8_t* sB = smem + KCH * kM * 16;        // KCH x 128 x 16
    __shared__ uint32_t s_tmem;
    __shared__ alignas(8) uint64_t s_bar;
    copy_image(sB, wimg, KCH * 128 * 16);
    fence_async_smem();
    cta_setup(&s_tmem, &s_bar, 1, 128);
    const uint32_t tmem = s_tmem;
    uint32_t phase = 0;
    const int lh = rs.rh / 4, lw = rs.rw / 4, ph = rs.rh / 2, pw = rs.rw / 2;
    const int nseg = (lw + kM - 1) / kM;
    const long long ntiles = (long long)rs.R * lh * nseg;
    const int t = threadIdx.x, warp = t >> 5;
    const uint32_t a0 = smem_addr(sA), b0 = smem_addr(sB);
    // A operand of a tile: this thread's pixel in every K chunk; the next tile's is loaded into
    // registers while the current tile's MMA and epilogue run
    uint4 pre[KCH];
    auto fetch = [&](long long tile) {
        const int seg = int(tile % nseg), y = int((tile / nseg) % lh), r = int(tile / ((long long)nseg * lh));
        const int xc = min(seg * kM + t, lw - 1);
#pragma unroll
        for (int c = 0; c < KCH; ++c) pre[c] = *cp_at(low, r, lh, y, KCH, c, lw, xc);
    };
    if (blockIdx.x < ntiles) fetch(blockIdx.x);
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        last_item(tile, ntiles);
        const int seg = int(tile % nseg), y = int((tile / nseg) % lh), r = int(tile / ((long long)nseg * lh));
        const int x = seg * kM + t, xc = min(x, lw - 1);
#pragma unroll
        for (int c = 0; c < KCH; ++c) *reinterpret_cast<uint4*>(sA + (c * kM + t) * 16) = pre[c];
        fence_async_smem();
        __syncthreads();
        if (t == 0) {
            fence_after_sync();
            constexpr uint32_t idesc = idesc_m128(128);
#pragma unroll
            for (int k = 0; k < KCH / 2; ++k) {
                const uint64_t a = sdesc(a0 + k * 2 * kM * 16, kM * 16, 128), b = sdesc(b0 + k * 2 * 128 * 16, 128 * 16, 128);
                if (FP8) mma_e4m3(tmem, a, b, idesc, k); else mma_f16(tmem, a, b, idesc, k);
            }
            commit(&s_bar);
        }
        // skip values of the tile's four output pixels, in flight during the MMA
        uint4 sk[4][4];
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int c = 0; c < 4; ++c) sk[p][c] = *cp_at(enc540, r, ph, 2 * y + (p >> 1), 4, c, pw, 2 * xc + (p & 1));
        if (tile + gridDim.x < ntiles) fetch(tile + gridDim.x);
        if (!mma_wait_all(&s_bar, phase, err)) break;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            float v[32];
            tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + p * 32, v);
            if (x < lw) {
                const int oy = 2 * y + (p >> 1), ox = 2 * x + (p & 1);
                const __half2* skh = reinterpret_cast<const __half2*>(sk[p]);
                epi_fma_leaky_cp(v, cp, p * 32, ep.slope, (FP8 || I8) ? ep.out_inv : 1.f);
                if (FP8) {   // K8: requantise to e4m3 at 1/s7, dequantise
#pragma unroll
                    for (int n = 0; n < 32; n += 4) {
                        float q[4];
                        e4m3x4_to_f32(e4m3x4(v[n], v[n + 1], v[n + 2], v[n + 3]), q);
#pragma unroll
                        for (int j = 0; j < 4; ++j) v[n + j] = q[j] * ep.out_deq;
                    }
                }
                if (I8) {   // int8 code at 1/s7, then code * s7 + skip in one rounding (int8_kernels.cuh:56-59)
#pragma unroll
                    for (int n = 0; n < 32; n += 2) {
                        const float2 sk = __half22float2(skh[n / 2]);
                        v[n] = fmaf(s8_code(v[n]), ep.out_deq, sk.x);
                        v[n + 1] = fmaf(s8_code(v[n + 1]), ep.out_deq, sk.y);
                    }
                } else {
#pragma unroll
                    for (int n = 0; n < 32; n += 2) {   // + the f16 skip
                        const float2 a = __fadd2_rn(make_float2(v[n], v[n + 1]), __half22float2(skh[n / 2]));
                        v[n] = a.x;
                        v[n + 1] = a.y;
                    }
                }
                uint4 o[4];
                pack_f16x32(v, o);
#pragma unroll
                for (int c = 0; c < 4; ++c) *cp_at(dec, r, ph, oy, 4, c, pw, ox) = o[c];
            }
        }
        fence_before_sync();
        __syncthreads();
    }
    cta_teardown(tmem, 128);
}

// ---- pipelined 3x3 layers ------------------------------------------------------------------
// Ring of NR input-row slots fed by TMA (thread 0), double-buffered TMEM accumulators.
// Per output row y of a (strip, band) work item:
//   wait MMA(y)  ->  TMA(row y+3) into the slot row y-1 used  ->  MMAs of row y+1 into the
//   other TMEM buffer  ->  epilogue of row y  ->  barrier.
// Every TMA issued is waited exactly once and every commit is waited exactly once, so the
// mbarrier parities stay in step across work items.
constexpr int kRing = 4;
// Output pixels per strip of the 3x3 kernels: the 128-pixel input window holds the strip and
// its one-pixel halo on either side; MMA rows 126 and 127 are computed and discarded.
constexpr int kConvStrip = kM - 2;

__device__ __forceinline__ uint8_t* align_smem(uint8_t* p) {
    const uint32_t a = smem_addr(p);
    return p + ((1024u - (a & 1023u)) & 1023u);
}

struct Ring {
    uint8_t* base;
    uint32_t base_addr;
    int slot_bytes;
    uint64_t* full;       // kRing barriers
    uint32_t phase = 0;   // bit s: parity of the next completion of slot s (issuing thread)
    uint32_t pending = 0; // bit s: a load into slot s has not been waited for
    __device__ static int slot(int row) { return (row + 4 * kRing) % kRing; }
    __device__ bool wait(int row, int* err) {
        const int s = slot(row);
        const bool ok = mbar_wait_bounded(&full[s], (phase >> s) & 1u, err, kErrTimeout);
        if (ok) {
            phase ^= 1u << s;
            pending &= ~(1u << s);
        }
        return ok;
    }
    // Abort path: wait (bounded) for loads still in flight before the CTA exits.
    __device__ void drain(int* err) {
        for (int s = 0; s < kRing; ++s)
            if (pending & (1u << s)) {
                mbar_wait_bounded(&full[s], (phase >> s) & 1u, err, kErrTimeout, 200000000LL);
                phase ^= 1u << s;
            }
        pending = 0;
    }
    __device__ uint32_t addr(int row) const { return base_addr + slot(row) * slot_bytes; }
};

// Grouped (2 x 32->32) 3x3 bottleneck layer, warp-specialised: warp 4 is the producer (TMA
// row loads and MMA issue, lane 0 issuing), warps 0-3 are the epilogue (warp w drains TMEM
// lanes 32w..32w+31).  The two groups (independent 32->32 convolutions) run in separate CTAs
// (even blockIdx: group 0, odd: group 1), each staging only its group's input channels and
// weights.  Output rows go in pairs, as in k_tc_refine_tail: input rows y and y+1 feed both
// output rows of a pair, so their MMAs have N = 64 over the adjacent weight blocks of tap
// rows ky and ky+1 (output row y+1 in TMEM columns 0-31 of the pair buffer, y in 32-63);
// rows y-1 and y+2 feed one output row each (N = 32).  The two sides meet only on mbarriers:
//   acc_full[b]  tcgen05.commit of a pair's MMAs into TMEM buffer b  -> epilogue, producer
//   acc_empty[b] one arrive per epilogue warp once it has read buffer b -> producer
// The producer issues the taps of input rows y-1 and y before it waits for rows y+1 and y+2
// to land, and refills their slots with rows y+3 and y+4 once those taps completed
// (slot_free).
constexpr int kWsThreads = 160;

template <bool FP8, bool I8 = false>
__global__ void __launch_bounds__(kWsThreads, 4) k_tc_core(const __grid_constant__ CUtensorMap tin, RegionSet rs,
                                                        const uint8_t* __restrict__ wimg, EpiParams ep,
                                                        const ChannelParams<64> cp, void* __restrict__ out, int band,
                                                        int* err) {
    constexpr int ICH = FP8 ? 4 : 8;          // 16-byte chunks of the 64 input channels
    constexpr int CPG = ICH / 2;              // chunks per group (staged per row)
    constexpr int LBO = kM * 16, SLOT = CPG * LBO;   // a 128-pixel window per chunk
    constexpr int WBLK = 32 * 16, WLBO = 3 * WBLK;  // weights [kx][chunk][ky][32 rows][16 B]
    constexpr int BG = 9 * CPG * WBLK;        // bytes of one group's weights
    const int gb = int(blockIdx.x & 1);      // this CTA's group
    const long long cta = blockIdx.x >> 1, stride = gridDim.x >> 1;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = align_smem(smem_raw);   // TMA destinations: 1024-byte aligned ring
    uint8_t* sB = smem + kRing * SLOT;
    __shared__ uint32_t s_tmem;
    // ring slots, acc_full x2, slot_free (count 1), acc_empty x2 (count 4)
    __shared__ alignas(8) uint64_t s_bar[kRing + 5];
    uint64_t* acc_full = s_bar + kRing;
    uint64_t* slot_free = s_bar + kRing + 2;
    uint64_t* acc_empty = s_bar + kRing + 3;
    copy_image(sB, wimg + gb * BG, BG);
    if (threadIdx.x == 0)
        for (int b = 0; b < 2; ++b) mbar_init(&acc_empty[b], 4);
    fence_async_smem();
    cta_setup(&s_tmem, s_bar, kRing + 3, 128);
    const uint32_t tmem = s_tmem;
    const int lh = rs.rh / 4, lw = rs.rw / 4;
    const int nstrip = (lw + kConvStrip - 1) / kConvStrip, nband = (lh + band - 1) / band;
    const long long items = (long long)rs.R * nstrip * nband;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

    if (warp == 4) {
        // ---- producer: the whole warp follows the control flow, lane 0 issues ----
        const bool leader = lane == 0;
        const uint32_t b0 = smem_addr(sB);
        constexpr uint32_t idesc32 = idesc_m128(32), idesc64 = idesc_m128(64);
        Ring ring{smem, smem_addr(smem), SLOT, s_bar};
        uint32_t pairs = 0, seen = 0;   // pairs committed; pairs [0, seen) observed complete here
        bool ok = true;
        auto load = [&](int row, const StripBand& sb) {
            if (leader) {
                mbar_arrive_expect_tx(&s_bar[Ring::slot(row)], uint32_t(SLOT));
                tma_load_4d(smem + Ring::slot(row) * SLOT, &tin, 2 * (sb.x0 - 1), gb * CPG, row, sb.r, &s_bar[Ring::slot(row)]);
            }
            ring.pending |= 1u << Ring::slot(row);
        };
        // wait until the MMAs of pair q (and so of every earlier pair) have completed
        auto done = [&](uint32_t q) {
            const bool r = __all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[q & 1], (q >> 1) & 1, err, kErrTimeout));
            if (r) seen = q + 1;
            return r;
        };
        // the MMAs of input row `row` with the weights of tap row ky (and ky+1 when n64) into d
        auto taps = [&](uint32_t d, int row, int ky, bool n64, bool first) {
            const uint32_t a = ring.addr(row);
#pragma unroll
            for (int kx = 0; kx < 3; ++kx)
#pragma unroll
                for (int kk = 0; kk < CPG / 2; ++kk) {
                    const uint64_t ad = sdesc(a + 2 * kk * LBO + kx * 16, LBO, 128);
                    const uint64_t bd = sdesc(b0 + ((kx * CPG + 2 * kk) * 3 + ky) * WBLK, WLBO, 128);
                    const bool acc = !(first && kx == 0 && kk == 0);
                    if (FP8) mma_e4m3(d, ad, bd, n64 ? idesc64 : idesc32, acc);
                    else mma_f16(d, ad, bd, n64 ? idesc64 : idesc32, acc);
                }
        };
        for (long long item = cta; item < items && ok; item += stride) {
            last_item(item, items, stride);
            const StripBand sb = strip_band(item, nstrip, nband, band, lh, kConvStrip);
            // the previous item's last MMAs still read the ring: let them finish before refilling it
            if (seen < pairs && !(ok = done(pairs - 1))) break;
            for (int row = sb.y0 - 1; row <= min(sb.y0 + 2, sb.y1); ++row) load(row, sb);
            for (int row = sb.y0 - 1; row <= sb.y0 && ok; ++row) ok = __all_sync(0xffffffffu, ring.wait(row, err));
            for (int y = sb.y0; y < sb.y1 && ok; y += 2) {   // bands hold whole pairs
                const uint32_t p = pairs;
                const int b = p & 1;
                const uint32_t k = p >> 1;
                // buffer b free: its previous pair drained
                if (k > 0) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&acc_empty[b], (k - 1) & 1, err, kErrTimeout));
                if (!ok) break;
                fence_after_sync();
                const uint32_t d = tmem + b * 64;
                if (leader) {
                    taps(d, y, 0, true, true);              // [W0; W1] x row y: the first MMA initialises both rows
                    taps(d + 32, y - 1, 0, false, false);   // W0 x row y-1 -> output row y
                    commit(slot_free);                       // rows y-1 and y are read by nothing after these
                }
                __syncwarp();
                ok = __all_sync(0xffffffffu, ring.wait(y + 1, err));
                if (ok) ok = __all_sync(0xffffffffu, ring.wait(y + 2, err));
                if (ok) {
                    fence_after_sync();
                    if (leader) {
                        taps(d, y + 1, 1, true, false);    // [W1; W2] x row y+1
                        taps(d, y + 2, 2, false, false);   // W2 x row y+2 -> output row y+1
                    }
                }
                // commit even on abort, so that the teardown's wait covers every issued MMA
                if (leader) commit(&acc_full[b]);
                __syncwarp();
                ++pairs;
                // rows y+3, y+4 into the slots of rows y-1, y once their MMAs completed (issued
                // before the second half of the pair, so the wait is normally over at once)
                if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(slot_free, p & 1, err, kErrTimeout));
                if (!ok) break;
                if (y + 3 <= sb.y1) load(y + 3, sb);
                if (y + 4 <= sb.y1) load(y + 4, sb);
            }
        }
        // let copies and MMAs still in flight land before TMEM is released (MMAs complete in
        // issue order, so the last commit covers them all)
        ring.drain(err);
        if (seen < pairs)
            mbar_wait_bounded(&acc_full[(pairs - 1) & 1], ((pairs - 1) >> 1) & 1, err, kErrTimeout, 200000000LL);
    } else {
        // ---- epilogue warps: both rows of a pair ----
        uint32_t p = 0;
        bool ok = true;
        for (long long item = cta; item < items && ok; item += stride) {
            last_item(item, items, stride);
            const StripBand sb = strip_band(item, nstrip, nband, band, lh, kConvStrip);
            const int x = sb.x0 + t;
            for (int y0 = sb.y0; y0 < sb.y1; y0 += 2, ++p) {
                const int b = p & 1;
                ok = __all_sync(0xffffffffu, mbar_wait_idle(&acc_full[b], (p >> 1) & 1, err, kErrTimeout));
                if (!ok) break;
                fence_after_sync();
#pragma unroll
                for (int r = 0; r < 2; ++r) {   // output row y0 + r: TMEM columns 32 (r = 0) or 0 (r = 1)
                    float v[32];
                    tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + b * 64 + (1 - r) * 32, v);
                    if (r == 1) {   // every column read: hand the buffer back to the producer
                        fence_before_sync();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[b]);
                    }
                    // this CTA's group's channel vectors, from the constant bank (a uniform branch,
                    // so that each copy reads at constant offsets)
                    if (gb == 0) epi_fma_leaky_cp(v, cp, 0, ep.slope, (FP8 || I8) ? ep.out_inv : 1.f);
                    else epi_fma_leaky_cp(v, cp, 32, ep.slope, (FP8 || I8) ? ep.out_inv : 1.f);
                    if (I8) s8_codes32(v);
                    if (t < kConvStrip && x < lw) {
                        if (FP8) {
                            uint4 q[2];
                            pack_e4m3x32(v, q);
                            for (int c = 0; c < 2; ++c) *cp_at(out, sb.r, lh, y0 + r, ICH, gb * 2 + c, lw, x) = q[c];
                        } else {
                            uint4 q[4];
                            pack_f16x32(v, q);
                            for (int c = 0; c < 4; ++c) *cp_at(out, sb.r, lh, y0 + r, ICH, gb * 4 + c, lw, x) = q[c];
                        }
                    }
                }
            }
        }
    }
    cta_teardown(tmem, 128);
}

// refine_540 (3x3 32->64) + metadata_head (1x1 64->64), warp-specialised like k_tc_core, two
// output rows at a time.  Input rows y and y+1 feed both output rows y and y+1 with different
// taps, so their MMAs have N = 128: B = [W_ky; W_ky+1] (the weights are stored ky-innermost,
// so the two 64-row blocks are adjacent) writes output row y+1 to TMEM columns 0-63 and
// output row y to 64-127 of the pair's buffer.  Rows y-1 and y+2 feed one output row each
// (N = 64).  A pair takes 12 MMAs of N = 128 and 12 of N = 64 instead of 36 of N = 64, and the
// A operand of the shared rows is read once.
// The refine output (LeakyReLU, f16) goes to shared memory as the tail GEMM's A operand and
// never reaches HBM.  Warp 8 (producer) issues the pair's refine GEMMs into TMEM buffer
// pair&1 and refills the TMA ring.  Epilogue warpgroup w (warps 4w..4w+3) takes output row
// y + w of every pair: refine epilogue, then (after a barrier of its own 128 threads) one of
// its threads issues the row's tail GEMM into the same 64 columns, then the tail epilogue;
// the buffer returns to the producer when both warpgroups have read their tails.
// The tail epilogue writes clamped f16 coefficients in the head's layout
// meta[r][Y][2][X][8 f16]: LR pixel (Y, X) = (2y + i, 2x + j) takes channels
// (2i + j)*16 .. +16; optionally also the raw float32 head output (NHWC, 64 channels).
constexpr int kRefineThreads = 288;

// Packed rows of the region a refine work item covers: all of them when the raw head output is
// wanted (predict_coefficients returns the whole padded grid), otherwise only the row pairs
// that cover the region's core, the rows whose coefficients the head reads.  `span` is the
// number of rows the bands divide (the same on the host).
__host__ __device__ inline int refine_span(const RegionSet& rs, bool trim) {
    return trim ? min(rs.rh / 2, rs.core_h / 2 + 3) : rs.rh / 2;
}
__device__ __forceinline__ StripBand refine_item(long long item, const RegionSet& rs, int nstrip, int nband, int band,
                                                 bool trim, bool& skip) {
    StripBand s = strip_band(item, nstrip, nband, band, rs.rh / 2, kConvStrip);
    skip = false;
    if (trim) {
        const int4 core = rs.cores[s.r];
        const int py0 = (core.x >> 1) & ~1, py1 = min(rs.rh / 2, (((core.z + 1) >> 1) + 1) & ~1);
        s.y0 += py0;
        s.y1 = min(s.y0 + band, py1);
        skip = s.y0 >= py1;
    }
    return s;
}

// sign(a) xor sign(b) times min(|a|, |b|); with one NaN operand, the other's magnitude
__device__ __forceinline__ float min_xorsign_abs(float a, float b) {
    float r;
    asm("min.xorsign.abs.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Barrier among the 128 threads of epilogue warpgroup wg (ids 1, 2); returns whether any of them
// passed `v`, so an abort is taken by the whole warpgroup.
__device__ __forceinline__ bool warpgroup_sync_or(int wg, bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, 128, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}\n"
                 : "=r"(r) : "r"(uint32_t(v)), "r"(1 + wg) : "memory");
    return r != 0;
}

__global__ void __launch_bounds__(kRefineThreads, 2) k_tc_refine_tail(const __grid_constant__ CUtensorMap tin, RegionSet rs,
                                                               const uint8_t* __restrict__ wref,
                                                               const uint8_t* __restrict__ wtail,
                                                               const RefineBiases bias, float slope,
                                                               void* __restrict__ meta, float* __restrict__ raw,
                                                               int band, int* err) {
    constexpr int ICH = 4, LBO = kM * 16, SLOT = ICH * LBO;   // a 128-pixel window per chunk
    constexpr int BREF = 36 * 64 * 16, BTAIL = 8 * 64 * 16, A2 = 8 * kM * 16;
    constexpr int WBLK = 64 * 16, WLBO = 3 * WBLK;   // weights [kx][k4][ky][64 rows][16 B]
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = align_smem(smem_raw);   // TMA destinations: 1024-byte aligned ring
    uint8_t* sB = smem + kRing * SLOT;   // refine weights
    uint8_t* sT = sB + BREF;             // tail weights
    uint8_t* sA2 = sT + BTAIL;           // tail operands, one per warpgroup
    __shared__ uint32_t s_tmem;
    // ring slots, then per buffer b: ref_full, tail_full (count 1); slot_free (count 1); then
    // per buffer pair_empty (count 8: every epilogue warp)
    __shared__ alignas(8) uint64_t s_bar[kRing + 7];
    uint64_t* ref_full = s_bar + kRing;
    uint64_t* tail_full = s_bar + kRing + 2;
    uint64_t* slot_free = s_bar + kRing + 4;
    uint64_t* pair_empty = s_bar + kRing + 5;
    copy_image(sB, wref, BREF);
    copy_image(sT, wtail, BTAIL);
    if (threadIdx.x == 0)
        for (int i = kRing + 5; i < kRing + 7; ++i) mbar_init(&s_bar[i], 8);
    fence_async_smem();
    cta_setup(&s_tmem, s_bar, kRing + 5, 256);
    const uint32_t tmem = s_tmem;
    const int ph = rs.rh / 2, pw = rs.rw / 2;
    const bool trim = raw == nullptr;
    const int nstrip = (pw + kConvStrip - 1) / kConvStrip, nband = (refine_span(rs, trim) + band - 1) / band;
    const long long items = (long long)rs.R * nstrip * nband;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    constexpr uint32_t idesc64 = idesc_m128(64), idesc128 = idesc_m128(128);

    if (warp == 8) {
        // ---- producer: the whole warp follows the control flow, lane 0 issues ----
        const bool leader = lane == 0;
        const uint32_t b0 = smem_addr(sB);
        Ring ring{smem, smem_addr(smem), SLOT, s_bar};
        uint32_t pairs = 0, seen = 0;   // pairs committed; pairs [0, seen) observed complete here
        bool ok = true;
        auto load = [&](int row, const StripBand& sb) {
            if (leader) {
                mbar_arrive_expect_tx(&s_bar[Ring::slot(row)], uint32_t(SLOT));
                tma_load_4d(smem + Ring::slot(row) * SLOT, &tin, 2 * (sb.x0 - 1), 0, row, sb.r, &s_bar[Ring::slot(row)]);
            }
            ring.pending |= 1u << Ring::slot(row);
        };
        // wait until the refine MMAs of pair q (and so of every earlier pair) have completed
        auto done = [&](uint32_t q) {
            const bool r = __all_sync(0xffffffffu, mbar_wait_bounded(&ref_full[q & 1], (q >> 1) & 1, err, kErrTimeout));
            if (r) seen = q + 1;
            return r;
        };
        // the 6 MMAs of input row `row` with the weights of tap row ky (and ky+1 when n128) into d
        auto taps = [&](uint32_t d, int row, int ky, bool n128, bool first) {
            const uint32_t a = ring.addr(row);
#pragma unroll
            for (int kx = 0; kx < 3; ++kx)
#pragma unroll
                for (int kk = 0; kk < 2; ++kk)
                    mma_f16(d, sdesc(a + 2 * kk * LBO + kx * 16, LBO, 128),
                            sdesc(b0 + ((kx * 4 + 2 * kk) * 3 + ky) * WBLK, WLBO, 128), n128 ? idesc128 : idesc64,
                            !(first && kx == 0 && kk == 0));
        };
        for (long long item = blockIdx.x; item < items && ok; item += gridDim.x) {
            last_item(item, items);
            bool skip;
            const StripBand sb = refine_item(item, rs, nstrip, nband, band, trim, skip);
            if (skip) continue;   // uniform across the CTA
            // the previous item's last MMAs still read the ring: let them finish before refilling it
            if (seen < pairs && !(ok = done(pairs - 1))) break;
            for (int row = sb.y0 - 1; row <= min(sb.y0 + 2, sb.y1); ++row) load(row, sb);
            for (int row = sb.y0 - 1; row <= sb.y0 && ok; ++row) ok = __all_sync(0xffffffffu, ring.wait(row, err));
            for (int y = sb.y0; y < sb.y1 && ok; y += 2) {   // bands hold whole pairs
                const uint32_t p = pairs;
                const int b = p & 1;
                const uint32_t k = p >> 1;
                // buffer b free: both warpgroups read the tails of pair p-2
                if (k > 0) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&pair_empty[b], (k - 1) & 1, err, kErrTimeout));
                if (!ok) break;
                fence_after_sync();
                const uint32_t d = tmem + b * 128;
                if (leader) {
                    taps(d, y, 0, true, true);        // [W0; W1] x row y: the first MMA initialises both rows
                    taps(d + 64, y - 1, 0, false, false);   // W0 x row y-1 -> output row y
                    commit(slot_free);                 // rows y-1 and y are read by nothing after these
                }
                __syncwarp();
                ok = __all_sync(0xffffffffu, ring.wait(y + 1, err));
                if (ok) ok = __all_sync(0xffffffffu, ring.wait(y + 2, err));
                if (ok) {
                    fence_after_sync();
                    if (leader) {
                        taps(d, y + 1, 1, true, false);   // [W1; W2] x row y+1
                        taps(d, y + 2, 2, false, false);  // W2 x row y+2 -> output row y+1
                    }
                }
                // commit even on abort, so that the teardown's wait covers every issued MMA
                if (leader) commit(&ref_full[b]);
                __syncwarp();
                ++pairs;
                // rows y+3, y+4 into the slots of rows y-1, y once their MMAs completed (issued
                // twelve MMAs ago, so the wait is normally over at once)
                if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(slot_free, p & 1, err, kErrTimeout));
                if (!ok) break;
                if (y + 3 <= sb.y1) load(y + 3, sb);
                if (y + 4 <= sb.y1) load(y + 4, sb);
            }
        }
        // let copies and MMAs still in flight land before TMEM is released (MMAs complete in
        // issue order, so the last commit covers them all)
        ring.drain(err);
        if (seen < pairs)
            mbar_wait_bounded(&ref_full[(pairs - 1) & 1], ((pairs - 1) >> 1) & 1, err, kErrTimeout, 200000000LL);
    } else {
        // ---- epilogue: warpgroup wg takes output row y + wg of every pair ----
        // Loop exits are decided only by the warpgroup's barrier vote (`live`), never by one
        // warp alone, so no warp can leave while the others wait at the warpgroup barrier.
        const int wg = warp >> 2, tq = t & 127;
        const uint32_t lrow = uint32_t(32 * (warp & 3)) << 16;
        const uint32_t half = wg == 0 ? 64 : 0;   // TMEM columns of this warpgroup's row in a pair buffer
        uint8_t* a2 = sA2 + wg * A2;
        const uint32_t a2addr = smem_addr(a2), t0 = smem_addr(sT);
        uint32_t p = 0, tail_phase = 0;
        bool live = true, bad = false;   // bad: a wait of this warp expired (voted at the next barrier)
        bool tail_pend = false;          // thread tq == 0 committed a tail not yet observed
        for (long long item = blockIdx.x; item < items && live; item += gridDim.x) {
            last_item(item, items);
            bool skip;
            const StripBand sb = refine_item(item, rs, nstrip, nband, band, trim, skip);
            if (skip) continue;
            const int x = sb.x0 + tq;
            for (int y0 = sb.y0; y0 < sb.y1 && live; y0 += 2, ++p) {
                const int b = p & 1, y = y0 + wg;
                const uint32_t col = tmem + lrow + b * 128 + half;
                // refine epilogue -> tail operand of this row
                if (!bad) bad = !__all_sync(0xffffffffu, mbar_wait_idle(&ref_full[b], (p >> 1) & 1, err, kErrTimeout));
                if (!bad) {
                    fence_after_sync();
                    float vr[2][32];
                    tmem_ld32x2(col, col + 32, vr[0], vr[1]);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {   // leaky(v + bias), as epi_add_leaky
                            const float2 a = __fadd2_rn(make_float2(vr[h][2 * i], vr[h][2 * i + 1]),
                                                        make_float2(bias.refine[h * 32 + 2 * i], bias.refine[h * 32 + 2 * i + 1]));
                            const float2 n = __fmul2_rn(a, make_float2(slope, slope));
                            vr[h][2 * i] = fmaxf(a.x, n.x);
                            vr[h][2 * i + 1] = fmaxf(a.y, n.y);
                        }
                        uint4 q[4];
                        pack_f16x32(vr[h], q);
#pragma unroll
                        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(a2 + ((h * 4 + c) * kM + tq) * 16) = q[c];
                    }
                    fence_async_smem();
                }
                // the whole operand is written, every warp's refine columns are read (the tail
                // overwrites them) and every warp's previous tail read is done
                fence_before_sync();
                if (warpgroup_sync_or(wg, bad)) {
                    live = false;
                    break;
                }
                if (tq == 0) {
                    fence_after_sync();
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16(tmem + b * 128 + half, sdesc(a2addr + kk * 2 * kM * 16, kM * 16, 128),
                                sdesc(t0 + kk * 2 * 64 * 16, 64 * 16, 128), idesc64, kk > 0);
                    commit(&tail_full[wg]);
                    tail_pend = true;
                }
                // tail epilogue of this row
                bad = !__all_sync(0xffffffffu, mbar_wait_idle(&tail_full[wg], tail_phase, err, kErrTimeout));
                if (bad) continue;
                tail_phase ^= 1u;
                tail_pend = false;
                fence_after_sync();
                float vt[2][32];
                tmem_ld32x2(col, col + 32, vt[0], vt[1]);
                fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&pair_empty[b]);   // this warp's part of the buffer is read
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float (&v)[32] = vt[h];
                    if (tq < kConvStrip && x < pw) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {   // v + bias, as epi_add
                            const float2 a = __fadd2_rn(make_float2(v[2 * i], v[2 * i + 1]),
                                                        make_float2(bias.tail[h * 32 + 2 * i], bias.tail[h * 32 + 2 * i + 1]));
                            v[2 * i] = a.x;
                            v[2 * i + 1] = a.y;
                        }
                        if (raw) {
                            float* rp = raw + (((size_t)sb.r * ph + y) * pw + x) * 64 + h * 32;
#pragma unroll
                            for (int n = 0; n < 32; ++n) rp[n] = v[n];
                        }
#pragma unroll
                        for (int n = 0; n < 32; n += 2) {   // coefficient_clamp
                            // v if |v| <= 2, else sign(v) * min(2 + 0.05 (|v| - 2), 2.5).  For |v| <= 2
                            // the soft term is >= |v| (also after rounding), so one min covers both
                            // cases.  The soft term is monotone and reaches exactly 2.5 at |v| = 12
                            // (fma(0.05f, 10, 2) rounds to 2.5f), so min(soft(|v|), 2.5) =
                            // soft(min(|v|, 12)).  min.xorsign.abs(v, c) = sign(v) * min(|v|, c) for
                            // c > 0; a NaN v gives min(NaN, 12) = 12, so sign * 2.5, as the
                            // reference's select does
                            const float2 soft = __ffma2_rn(make_float2(0.05f, 0.05f),
                                                           __fadd2_rn(make_float2(fminf(fabsf(v[n]), 12.f),
                                                                                  fminf(fabsf(v[n + 1]), 12.f)),
                                                                      make_float2(-2.f, -2.f)),
                                                           make_float2(2.f, 2.f));
                            v[n] = min_xorsign_abs(v[n], soft.x);
                            v[n + 1] = min_xorsign_abs(v[n + 1], soft.y);
                        }
                        uint4 q[4];
                        pack_f16x32(v, q);
                        // LR pixels (2y + h, 2x) and (2y + h, 2x + 1) are adjacent in each chunk
                        // plane: chunk c of both in one 32-byte store (2x is even, rw a multiple of 32)
#pragma unroll
                        for (int c = 0; c < 2; ++c)
                            st_global_2x16(cp_at(meta, sb.r, rs.rh, 2 * y + h, 2, c, rs.rw, 2 * x), q[c], q[2 + c]);
                    }
                }
            }
        }
        if (tq == 0 && tail_pend)   // abort path: the committed tail lands before TMEM is released
            mbar_wait_bounded(&tail_full[wg], tail_phase, err, kErrTimeout, 200000000LL);
    }
    cta_teardown(tmem, 256);
}

// ---- reconstruction head -------------------------------------------------------------------
// Work item: a strip of PX * 128 LR pixels of a region's core rectangle and a band of rows.
// Thread t owns pixels x0 + t + 128 i (tile i < PX) of every row of the band.  Per row, one
// elected thread loads the tiles' clamped f16 coefficients with TMA row-window loads (128
// pixels x 2 chunks each) and, per tile, issues
//   D[px][tap*4 + phase] = sum_k c_k * basis_hi + sum_k c_k * basis_lo + base_hi + base_lo
// (three K = 16 MMAs; the FP32 bank is split into two f16 terms, so the filters keep FP32-level
// accuracy) into that tile's 128 TMEM columns.  Each thread then applies its pixels' 25 x 4
// weights to their 5 x 5 RGB neighbourhoods on the CUDA cores.  Source rows slide through an
// 8-row ring in shared memory, converted once per strip and stored as (s[x], s[x+1]) pairs that
// feed packed f32x2 FMAs directly; the next row's coefficients arrive by TMA and its new source
// row is loaded into registers while the current row computes; the TMEM loads of one column
// group are issued before the FMAs of the previous one.  Several CTAs share an SM, so one CTA's
// MMA and TMA waits hide behind the others' FMAs.  The kernel is specialised on the source
// (uint8 HWC or float32 CHW) and destination (uint8 HWC or float32 CHW) formats.
constexpr int kHeadRing = 8;
constexpr int kHeadBCH = 2 * 128 * 16;             // one B operand: N = 128 rows, 2 K chunks
constexpr int kHeadTile = 2 * kM * 16;             // one tile's A operand: 2 K chunks x 128 rows (one TMA box)
// PX pixels per thread: a strip of PX * 128 LR pixels, PX * 128 TMEM columns per CTA
constexpr int head_strip(int px) { return px * kM; }
constexpr int head_tw(int px) { return px * kM + 4; }   // source columns of a strip (2 halo columns each side)
constexpr int head_smem(int px) {
    return 1024 + 2 * px * kHeadTile + 3 * kHeadBCH + kM * 16 * 2 + kHeadRing * 3 * (head_tw(px) + 1) * 8;
}

// floor(clamp(v, 0, 1) * 255 + 0.5) with separate multiply and add (runtime.py:24-25 in
// float32), for two values at once (packed f32x2 arithmetic rounds each lane as the scalar
// operation does).  The sum lies in [0.5, 255.5]; adding 2^23 with round-down leaves
// floor(sum) in the low mantissa bits, so byte 0 of each result is the output code.
__device__ __forceinline__ uint2 u8_code_bits2(float a, float b) {
    const float2 m = __fmul2_rn(make_float2(__saturatef(a), __saturatef(b)), make_float2(255.f, 255.f));
    const float2 f = __fadd2_rd(__fadd2_rn(m, make_float2(0.5f, 0.5f)), make_float2(8388608.f, 8388608.f));
    return make_uint2(__float_as_uint(f.x), __float_as_uint(f.y));
}

template <int PX, bool SRC_U8, bool DST_U8>
__global__ void __launch_bounds__(kThreads, PX == 1 ? 4 : 2) k_tc_head(const __grid_constant__ CUtensorMap tcoef, SrcDesc src,
                                                         RegionSet rs, DstDesc dst, const uint8_t* __restrict__ bimg,
                                                         int band, int* nonfinite, int* err) {
    constexpr int kHeadStrip = head_strip(PX), kHeadTW = head_tw(PX), kHeadABytes = PX * kHeadTile;
    constexpr uint32_t kCols = 128 * PX;                  // TMEM columns: 128 per tile
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = align_smem(smem_raw);
    uint8_t* sA = smem;                                   // [2 rows][PX tiles][2 chunks][128][16 B] (TMA)
    uint8_t* sB = smem + 2 * kHeadABytes;                 // basis hi, basis lo, base
    uint8_t* sOnes = sB + 3 * kHeadBCH;                   // [2 chunks][128][16 B]
    // source ring: per slot and channel the pairs (s[x], s[x+1]) of adjacent columns, so a
    // horizontal tap pair is one 8-byte load that feeds packed f32x2 FMAs directly.  Each row
    // starts with one spare pair, the target of column 0's second half, so puts need no test.
    float2 (*s_pair)[3][kHeadTW + 1] = reinterpret_cast<float2 (*)[3][kHeadTW + 1]>(sOnes + 2 * kM * 16);
    __shared__ float s_lut[256];
    __shared__ uint32_t s_tmem;
    __shared__ alignas(8) uint64_t s_bar[3];              // MMA round done; coefficient rows of A buffer 0, 1
    copy_image(sB, bimg, 3 * kHeadBCH);
    for (int i = threadIdx.x; i < 2 * kM; i += blockDim.x) {
        const uint32_t one2 = 0x3C003C00u;   // f16 1.0, 1.0
        *reinterpret_cast<uint4*>(sOnes + i * 16) = (i < kM) ? make_uint4(one2, 0, 0, 0) : make_uint4(0, 0, 0, 0);
    }
    if (SRC_U8) fill_lut(s_lut);
    fence_async_smem();
    cta_setup(&s_tmem, s_bar, 3, kCols);
    const uint32_t tmem = s_tmem;
    const int t = threadIdx.x, warp = t >> 5;
    const uint32_t lane = uint32_t(32 * warp) << 16;
    const int nstrip = (rs.core_w + kHeadStrip - 1) / kHeadStrip, nband = (rs.core_h + band - 1) / band;
    const long long items = (long long)rs.R * nstrip * nband;
    const uint32_t o0 = smem_addr(sOnes), b0 = smem_addr(sB), a0 = smem_addr(sA);
    // N = 112: the 100 weight columns of a tile; columns 112-119 take the tile's coefficients
    // (the MMAs' A operand, copied there from shared memory), 120-127 a constant ones operand
    // (its first two K entries 1) for the base term
    constexpr uint32_t idesc = idesc_m128(112);
    // Work beside the apply is spread over the warps: warp 1 issues the loads and MMAs, the last
    // four threads stage the four window columns beyond PX per thread.
    constexpr int kExtra = kHeadTW - PX * kThreads;
    const bool extra = t >= kThreads - kExtra;
    // strip column of source column j of this thread: t + 128 j, and for j = PX the extra column
    auto col_of = [&](int j) { return j < PX ? t + j * kThreads : PX * kThreads + t - (kThreads - kExtra); };
    const bool issuer = t == 32;
    if (issuer)
#pragma unroll
        for (int tile = 0; tile < PX; ++tile) tmem_cp_128x256b(tmem + tile * 128 + 120, sdesc(o0, kM * 16, 128));
    uint32_t mma_phase = 0, tma_phase = 0, tma_pend = 0;   // tma bits: per A buffer
    bool ok = true, mma_pend = false;
    // coefficient rows of row y into A buffer b: PX boxes of 128 pixels x 2 chunks
    auto load_coef = [&](int r, int y, int x0, int b) {
        mbar_arrive_expect_tx(&s_bar[1 + b], uint32_t(kHeadABytes));
#pragma unroll
        for (int h = 0; h < PX; ++h)
            tma_load_4d(sA + b * kHeadABytes + h * kHeadTile, &tcoef, 2 * (x0 + h * kM), 0, y, r, &s_bar[1 + b]);
        tma_pend |= 1u << b;
    };
    // MMA round of the row whose coefficients are (being) loaded into A buffer b.  On an expired
    // wait no MMA is issued, but the commit still arrives, so that no thread waits for it in vain.
    auto issue = [&](int b) {
        const uint32_t par = (tma_phase >> b) & 1u;
        const bool landed = mbar_try_wait(&s_bar[1 + b], par) || mbar_wait_bounded(&s_bar[1 + b], par, err, kErrTimeout);
        if (landed) {
            tma_phase ^= 1u << b;
            tma_pend &= ~(1u << b);
            fence_after_sync();
#pragma unroll
            for (int tile = 0; tile < PX; ++tile) {
                const uint32_t d = tmem + tile * 128;
                tmem_cp_128x256b(d + 112, sdesc(a0 + b * kHeadABytes + tile * kHeadTile, kM * 16, 128));
                mma_f16_ta(d, d + 112, sdesc(b0, 128 * 16, 128), idesc, 0);
                mma_f16_ta(d, d + 112, sdesc(b0 + kHeadBCH, 128 * 16, 128), idesc, 1);
                mma_f16_ta(d, d + 120, sdesc(b0 + 2 * kHeadBCH, 128 * 16, 128), idesc, 1);
            }
        }
        commit(&s_bar[0]);
        mma_pend = true;
        return landed;
    };

    for (long long item = blockIdx.x; item < items && ok; item += gridDim.x) {
        last_item(item, items);
        const int r = int(item / ((long long)nstrip * nband));
        const int bi = int((item / nstrip) % nband), si = int(item % nstrip);
        const int4 core = rs.cores[r];
        const int y0 = core.x + bi * band, x0 = core.y + si * kHeadStrip;
        if (y0 >= core.z || x0 >= core.w) continue;            // uniform across the CTA
        const int y1 = min(y0 + band, core.z);
        const int4 reg = rs.regions[r];
        // this thread's source columns (col_of(j)), clamped once per item: region replicate
        // padding, then the frame's
        int scol[PX + 1];
#pragma unroll
        for (int j = 0; j <= PX; ++j)
            scol[j] = clampi(reg.z + clampi(x0 - 2 + col_of(j), 0, rs.rw - 1) - src.pad_x, 0, src.W - 1);
        const size_t plane = size_t(src.H) * src.W;
        const uint8_t* sfu8 = static_cast<const uint8_t*>(src.ptr) + size_t(reg.x) * plane * 3;
        const float* sff = static_cast<const float*>(src.ptr) + size_t(reg.x) * plane * 3;
        auto src_row = [&](int row) {   // element offset of the frame row that region row `row` reads
            const int sy = clampi(reg.y + clampi(row, 0, rs.rh - 1) - src.pad_y, 0, src.H - 1);
            return size_t(sy) * src.W;
        };
        auto src_raw = [&](size_t ro, int j) -> uint3 {
            if (SRC_U8) {
                const uint8_t* p = sfu8 + (ro + scol[j]) * 3;
                return make_uint3(p[0], p[1], p[2]);
            }
            const float* p = sff + ro + scol[j];
            return make_uint3(__float_as_uint(p[0]), __float_as_uint(p[plane]), __float_as_uint(p[2 * plane]));
        };
        auto slot = [&](int row) { return (row - y0 + 2) & (kHeadRing - 1); };
        auto put = [&](int row, int j, uint3 raw) {   // column col: first of pair col, second of pair col - 1
            float v[3];
            if (SRC_U8) {
                v[0] = s_lut[raw.x]; v[1] = s_lut[raw.y]; v[2] = s_lut[raw.z];
            } else {
                v[0] = __uint_as_float(raw.x); v[1] = __uint_as_float(raw.y); v[2] = __uint_as_float(raw.z);
            }
            float* ps = &s_pair[slot(row)][0][col_of(j) + 1].x;
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                ps[ch * 2 * (kHeadTW + 1)] = v[ch];
                ps[ch * 2 * (kHeadTW + 1) - 1] = v[ch];
            }
        };
        // output: frame base and this thread's first output column of each tile
        const int oxA = 2 * (reg.z + x0 + t - dst.pad_x);

        // prologue: source rows y0-2 .. y0+2, coefficients of y0, MMA(y0)
        if (issuer) load_coef(r, y0, x0, 0);
        for (int row = y0 - 2; row <= y0 + 2; ++row) {
            const size_t ro = src_row(row);
#pragma unroll
            for (int j = 0; j < PX; ++j) put(row, j, src_raw(ro, j));
            if (extra) put(row, PX, src_raw(ro, PX));
        }
        __syncthreads();
        if (issuer) ok = issue(0);
        for (int y = y0; y < y1; ++y) {
            const int b = (y - y0) & 1;
            // prefetch: next row's coefficients (TMA) and source row y+3 (registers)
            const bool next = y + 1 < y1;
            uint3 pre[PX + 1] = {};
            if (next) {
                if (issuer) load_coef(r, y + 1, x0, b ^ 1);
                const size_t ro = src_row(y + 3);
#pragma unroll
                for (int j = 0; j < PX; ++j) pre[j] = src_raw(ro, j);
                if (extra) pre[PX] = src_raw(ro, PX);
            }
            if (!mbar_try_wait(&s_bar[0], mma_phase) && !mbar_wait_bounded(&s_bar[0], mma_phase, err, kErrTimeout)) ok = false;
            else {
                mma_phase ^= 1u;
                mma_pend = false;
            }
            fence_after_sync();
            // the window rows y-2 .. y+2 of this row, one ring slot each
            const float2(*rows[5])[kHeadTW + 1];
#pragma unroll
            for (int ky = 0; ky < 5; ++ky) rows[ky] = s_pair[slot(y - 2 + ky)];
            const int oy = 2 * (reg.y + y - dst.pad_y);
            const size_t orow_bytes = size_t(dst.OW) * 3;   // uint8 destination: this row pair's first byte
            uint8_t* orow = static_cast<uint8_t*>(dst.ptr) + (size_t(reg.x) * dst.OH + oy) * orow_bytes;
            // apply the 25 x 4 filter weights of both pixels, interleaved (two independent sets of
            // accumulator chains per TMEM wait).  acc[tile][p][ch] is a pair of partial sums (taps
            // with even kx and the fifth column | taps with odd kx); TMEM columns of a tile: tap
            // pairs (ky, 0|1) and (ky, 2|3) at (ky*2 + j)*8 + phase*2 + lane, then (ky, 4) at
            // 80 + ky*4 + phase
            float2 acc[PX][4][3];
#pragma unroll
            for (int tile = 0; tile < PX; ++tile)
#pragma unroll
                for (int p = 0; p < 4; ++p)
#pragma unroll
                    for (int ch = 0; ch < 3; ++ch) acc[tile][p][ch] = make_float2(0.f, 0.f);
            const uint32_t tcol = tmem + lane;
            // weights in four column groups per tile (0-31, 32-63, 64-95, 96-99); the loads of
            // group q+1 are issued before the FMAs of group q, so their latency hides behind them
            uint32_t wr[2][PX][32];   // [group parity][tile][column]
#pragma unroll
            for (int tile = 0; tile < PX; ++tile) tmem_ld_x32(tcol + tile * 128, wr[0][tile]);
            tmem_wait_ld();
#pragma unroll
            for (int tile = 0; tile < PX; ++tile) tmem_regs_ready(wr[0][tile]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
#pragma unroll
                for (int tile = 0; tile < PX; ++tile) {
                    if (q + 1 < 3) tmem_ld_x32(tcol + tile * 128 + (q + 1) * 32, wr[(q + 1) & 1][tile]);
                    else if (q + 1 == 3) tmem_ld_x4(tcol + tile * 128 + 96, wr[1][tile]);
                }
                const uint32_t(&wu)[PX][32] = wr[q & 1];
#pragma unroll
                for (int i = 0; i < (q < 3 ? 32 : 4); ++i) {
                    const int n = q * 32 + i;
                    if (n < 80 && i % 8 == 0) {   // tap pair (ky, 2j), (ky, 2j+1): 12 packed FMAs per pixel
                        const int pair = n / 8, ky = pair / 2, j = pair % 2;
#pragma unroll
                        for (int ch = 0; ch < 3; ++ch)
#pragma unroll
                            for (int tile = 0; tile < PX; ++tile) {
                                const float2 sv = rows[ky][ch][1 + t + tile * kM + 2 * j];
#pragma unroll
                                for (int p = 0; p < 4; ++p)
                                    acc[tile][p][ch] = __ffma2_rn(
                                        sv, make_float2(__uint_as_float(wu[tile][i + 2 * p]), __uint_as_float(wu[tile][i + 2 * p + 1])),
                                        acc[tile][p][ch]);
                            }
                    } else if (n >= 80 && n < 100 && (n - 80) % 4 == 0) {   // tap (ky, 4): 12 FMAs per pixel
                        const int ky = (n - 80) / 4;
#pragma unroll
                        for (int ch = 0; ch < 3; ++ch)
#pragma unroll
                            for (int tile = 0; tile < PX; ++tile) {
                                const float sv = rows[ky][ch][1 + t + tile * kM + 4].x;
#pragma unroll
                                for (int p = 0; p < 4; ++p)
                                    acc[tile][p][ch].x = fmaf(sv, __uint_as_float(wu[tile][i + p]), acc[tile][p][ch].x);
                            }
                    }
                }
                if (q + 1 < 4) {
                    tmem_wait_ld();
#pragma unroll
                    for (int tile = 0; tile < PX; ++tile) tmem_regs_ready(wr[(q + 1) & 1][tile]);
                }
            }
#pragma unroll
            for (int tile = 0; tile < PX; ++tile) {
                float out[4][3];
#pragma unroll
                for (int p = 0; p < 4; ++p)
#pragma unroll
                    for (int ch = 0; ch < 3; ++ch) out[p][ch] = acc[tile][p][ch].x + acc[tile][p][ch].y;
                if (x0 + tile * kM + t < core.w) {
                    // One test for all twelve values: a non-finite term makes the sum non-finite.  Only
                    // float sources can make one: with uint8 sources every tap value lies in [0, 1]
                    // and every filter weight is finite (clamped coefficients times a finite bank).
                    if (!SRC_U8) {
                        float2 all = __fadd2_rn(make_float2(out[0][0], out[0][1]), make_float2(out[0][2], out[1][0]));
                        all = __fadd2_rn(all, __fadd2_rn(make_float2(out[1][1], out[1][2]), make_float2(out[2][0], out[2][1])));
                        all = __fadd2_rn(all, __fadd2_rn(make_float2(out[2][2], out[3][0]), make_float2(out[3][1], out[3][2])));
                        if (!isfinite(all.x + all.y)) atomicOr(nonfinite, 1);
                    }
                    const int ox = oxA + tile * 2 * kM;
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        if (!DST_U8) {
                            float* o = static_cast<float*>(dst.ptr) + (size_t(reg.x) * 3 * dst.OH + oy + i) * dst.OW + ox;
                            const size_t chs = size_t(dst.OH) * dst.OW;
#pragma unroll
                            for (int ch = 0; ch < 3; ++ch)
                                *reinterpret_cast<float2*>(o + ch * chs) = make_float2(out[2 * i][ch], out[2 * i + 1][ch]);
                        } else {
                            // bytes r0 g0 b0 r1 g1 b1 of the two output pixels (phases 2i, 2i+1), as
                            // three 16-bit words (2-byte aligned: the row offset is a multiple of 6)
                            const uint2 q01 = u8_code_bits2(out[2 * i][0], out[2 * i][1]);
                            const uint2 q23 = u8_code_bits2(out[2 * i][2], out[2 * i + 1][0]);
                            const uint2 q45 = u8_code_bits2(out[2 * i + 1][1], out[2 * i + 1][2]);
                            unsigned short* o = reinterpret_cast<unsigned short*>(orow + i * orow_bytes + size_t(ox) * 3);
                            // streaming stores: the frame is read back only by the host copy
                            __stcs(o, (unsigned short)__byte_perm(q01.x, q01.y, 0x0040));
                            __stcs(o + 1, (unsigned short)__byte_perm(q23.x, q23.y, 0x0040));
                            __stcs(o + 2, (unsigned short)__byte_perm(q45.x, q45.y, 0x0040));
                        }
                    }
                }
            }
            // source row y+3 into the ring (read after this row's barrier)
            if (next) {
#pragma unroll
                for (int j = 0; j < PX; ++j) put(y + 3, j, pre[j]);
                if (extra) put(y + 3, PX, pre[PX]);
            }
            fence_before_sync();
            if (__syncthreads_or(!ok)) {
                ok = false;
                break;
            }
            if (issuer && next && !issue(b ^ 1)) ok = false;   // voted at the next row's barrier
        }
    }
    // abort path: let in-flight copies and MMAs land before TMEM and shared memory are released
    if (issuer) {
        if (mma_pend) mbar_wait_bounded(&s_bar[0], mma_phase, err, kErrTimeout, 200000000LL);
#pragma unroll
        for (int b = 0; b < 2; ++b)
            if (tma_pend & (1u << b)) mbar_wait_bounded(&s_bar[1 + b], (tma_phase >> b) & 1u, err, kErrTimeout, 200000000LL);
    }
    cta_teardown(tmem, kCols);
}

// ---- fused refine_540 + metadata_head + reconstruction head ---------------------------------
// One kernel from dec540 to the output frames: the clamped coefficients of a packed row go from
// the tail epilogue into shared memory as the head's A operands and never reach HBM.
// Eight warps, two warpgroups, one CTA per SM (all 512 TMEM columns); with no producer warp each
// thread may hold 255 registers.  Warpgroup wg takes packed row y + wg of every row pair: the
// refine epilogue, tail MMA and tail epilogue of k_tc_refine_tail, then the reconstruction of
// the row.  Lane tq holds packed pixel x = x0 + tq, whose four LR pixels (2y + i, 2x + j) make
// four tiles of 128 pixels: the A row of tile (i, j) is the lane's tail channels
// (2i + j)*16 .. +16, i.e. the 16 coefficients of LR pixel (2y + i, 2x + j).  The filter-mix
// MMAs of k_tc_head build each tile's 100 weights in two halves (columns 0-63 and 64-111 of the
// tile's layout: tap pairs of rows 0-3, then tap pairs of row 4 and the fifth column), eight
// halves per row.  Each warpgroup owns three 64-column TMEM buffers (128 + 192 wg); once every
// thread of the warpgroup has loaded half s, half s + 3 of the row is issued into its buffer, so
// each MMA runs under the FMAs of the halves before it.  Weights, accumulation order and output
// rounding are k_tc_head's, so the frames equal the unfused pair's bit for bit.
// Thread 0 also does the producer's work: dec540 rows (TMA) through a ring of six row slots, two
// pairs ahead, and the refine MMAs of the next pair (one pair buffer, TMEM columns 0-127) in four
// groups of six, the first once both warpgroups have read their tails (pair_empty), each issued
// after the head MMAs of a tile so that they queue behind them.
// LR source rows (region- then frame-clamped, converted to float once per strip) slide through
// a ring of 12 rows shared by both warpgroups: a pair reads 8 (2y - 2 .. 2y + 5) while the
// next pair's 4 new rows are fetched into registers and stored at the end of the pair; one
// barrier of both warpgroups per pair publishes them.  Each (row, channel) is stored twice, E =
// s[0..] and O = s[1..] (ring column c = LR column 2 x0 - 2 + c), so the horizontal tap pairs
// of an even pixel are the float2 E[tq + jj] and those of an odd pixel O[tq + jj]: a warp reads
// consecutive 8-byte pairs, free of bank conflicts.
// Work items: (region, strip of kConvStrip packed columns, band of packed rows) over the packed
// rectangle that covers the region's core, its rows rounded out to whole pairs.
constexpr int kFusedThreads = 256;
constexpr int kFusedRing = 6;             // dec540 row slots
constexpr int kSrcRing = 12;              // LR source rows in the ring
constexpr int kSrcCols = 2 * kM + 5;      // ring columns a strip reads (2 x0 - 2 .. 2 x0 + 258)
constexpr int kSrcArr = 264;              // floats per (row, channel) array E or O
constexpr int kFusedBytes = 1024 + kFusedRing * 4 * kM * 16 + 36 * 64 * 16 + 8 * 64 * 16 + 2 * 8 * kM * 16 +
                            3 * kHeadBCH + 2 * kM * 16 + 2 * 64 * 4 + 256 * 4 + kSrcRing * 3 * 2 * kSrcArr * 4;
static_assert(kFusedBytes <= 220 * 1024, "fused kernel's shared memory");

struct FusedItem {
    int r, x0, y0, y1, px1;
    int4 core;
    bool skip;
};
__device__ __forceinline__ FusedItem fused_item(long long item, const RegionSet& rs, int nstrip, int nband,
                                                int band) {
    FusedItem f;
    f.r = int(item / ((long long)nstrip * nband));
    const int bi = int((item / nstrip) % nband), si = int(item % nstrip);
    f.core = rs.cores[f.r];
    const int py0 = (f.core.x >> 1) & ~1, py1 = min(rs.rh / 2, (((f.core.z + 1) >> 1) + 1) & ~1);
    f.px1 = (f.core.w + 1) >> 1;
    f.x0 = (f.core.y >> 1) + si * kConvStrip;
    f.y0 = py0 + bi * band;
    f.y1 = min(f.y0 + band, py1);
    f.skip = f.x0 >= f.px1 || f.y0 >= py1;
    return f;
}

// Barrier of both warpgroups (id 3, 256 threads); returns whether any thread passed `v`.
__device__ __forceinline__ bool epilogues_sync_or(bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 3, 256, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}\n"
                 : "=r"(r) : "r"(uint32_t(v)) : "memory");
    return r != 0;
}

template <bool SRC_U8, bool DST_U8>
__global__ void __launch_bounds__(kFusedThreads, 1) k_tc_refine_head(const __grid_constant__ CUtensorMap tin, RegionSet rs,
                                                              const uint8_t* __restrict__ wref,
                                                              const uint8_t* __restrict__ wtail,
                                                              const float* __restrict__ rbias,
                                                              const float* __restrict__ tbias, float slope,
                                                              const uint8_t* __restrict__ bimg, SrcDesc src,
                                                              DstDesc dst, int band, int nstrip, int nband,
                                                              int* nonfinite, int* err) {
    constexpr int ICH = 4, LBO = kM * 16, SLOT = ICH * LBO;
    constexpr int BREF = 36 * 64 * 16, BTAIL = 8 * 64 * 16, A2 = 8 * kM * 16;
    constexpr int WBLK = 64 * 16, WLBO = 3 * WBLK;
    constexpr int ROWF = 3 * 2 * kSrcArr;     // floats per source ring row: per channel E then O
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = align_smem(smem_raw);     // TMA destinations: 1024-byte aligned ring
    uint8_t* sB = smem + kFusedRing * SLOT;   // refine weights
    uint8_t* sT = sB + BREF;                  // tail weights
    uint8_t* sA2 = sT + BTAIL;                // per warpgroup: the tail's A operand, then the head's 4 tiles
    uint8_t* sHB = sA2 + 2 * A2;              // head B operands: basis hi, basis lo, base
    uint8_t* sOnes = sHB + 3 * kHeadBCH;      // [2 chunks][128][16 B]
    float* s_rb = reinterpret_cast<float*>(sOnes + 2 * kM * 16);
    float* s_tb = s_rb + 64;
    float* s_lut = s_tb + 64;
    float* s_src = s_lut + 256;               // [kSrcRing][3][E | O][kSrcArr]
    __shared__ uint32_t s_tmem;
    // dec540 slots, ref_full; per warpgroup tail_full, drain; per warpgroup and head buffer
    // head_full (all count 1); pair_empty (count 8: every warp, once it has read its tail)
    __shared__ alignas(8) uint64_t s_bar[kFusedRing + 12];
    uint64_t* ring_full = s_bar;
    uint64_t* ref_full = s_bar + kFusedRing;
    uint64_t* tail_full = s_bar + kFusedRing + 1;
    uint64_t* drain = s_bar + kFusedRing + 3;
    uint64_t* head_full = s_bar + kFusedRing + 5;
    uint64_t* pair_empty = s_bar + kFusedRing + 11;
    copy_image(sB, wref, BREF);
    copy_image(sT, wtail, BTAIL);
    copy_image(sHB, bimg, 3 * kHeadBCH);
    for (int i = threadIdx.x; i < 2 * kM; i += blockDim.x) {
        const uint32_t one2 = 0x3C003C00u;   // f16 1.0, 1.0
        *reinterpret_cast<uint4*>(sOnes + i * 16) = (i < kM) ? make_uint4(one2, 0, 0, 0) : make_uint4(0, 0, 0, 0);
    }
    if (threadIdx.x < 64) { s_rb[threadIdx.x] = rbias[threadIdx.x]; s_tb[threadIdx.x] = tbias[threadIdx.x]; }
    if (SRC_U8) fill_lut(s_lut);
    if (threadIdx.x == 0) mbar_init(pair_empty, 8);
    fence_async_smem();
    cta_setup(&s_tmem, s_bar, kFusedRing + 11, 512);
    const uint32_t tmem = s_tmem;
    const long long items = (long long)rs.R * nstrip * nband;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int wg = warp >> 2, tq = t & 127;
    const bool issuer = t == 0;                  // producer work, and warpgroup 0's tail and head MMAs
    const uint32_t lrow = uint32_t(32 * (warp & 3)) << 16;
    const uint32_t half = wg == 0 ? 64 : 0;   // TMEM columns of this warpgroup's row in the pair buffer
    uint8_t* a2 = sA2 + wg * A2;
    const uint32_t a2addr = smem_addr(a2), t0 = smem_addr(sT), hb0 = smem_addr(sHB), o0 = smem_addr(sOnes);
    const uint32_t b0 = smem_addr(sB), ring0 = smem_addr(smem);
    constexpr uint32_t idesc64 = idesc_m128(64), idesc128 = idesc_m128(128);
    // this warpgroup's three filter-weight buffers; half s of a row (tile s >> 1, half s & 1)
    // goes to buffer (hs + s) % 3, hs counting the halves of the warpgroup's earlier rows
    const uint32_t hcol = tmem + 128 + uint32_t(wg) * 192;
    const size_t plane = size_t(src.H) * src.W;
    uint32_t p = 0, tail_phase = 0, hs = 0, head_phase = 0;   // head_phase: bit per buffer
    uint32_t ring_phase = 0, ring_pend = 0;          // issuer: per dec540 slot
    // bad: a wait of this warp expired; pbad: one of the issuer's producer waits expired; dead:
    // the warpgroup voted to stop.  All three enter every vote.
    bool live = true, bad = false, dead = false, pbad = false;

    // ---- producer work (issuer only) ----
    auto slot_of = [](int row) { return (row + kFusedRing) % kFusedRing; };   // rows >= -1
    auto load_row = [&](int row, const FusedItem& fi) {
        const int sl = slot_of(row);
        mbar_arrive_expect_tx(&ring_full[sl], uint32_t(SLOT));
        tma_load_4d(smem + sl * SLOT, &tin, 2 * (fi.x0 - 1), 0, row, fi.r, &ring_full[sl]);
        ring_pend |= 1u << sl;
    };
    auto wait_row = [&](int row) {
        const int sl = slot_of(row);
        if (!(ring_pend & (1u << sl))) return true;   // already observed
        const bool ok = mbar_wait_bounded(&ring_full[sl], (ring_phase >> sl) & 1u, err, kErrTimeout);
        if (ok) {
            ring_phase ^= 1u << sl;
            ring_pend &= ~(1u << sl);
        }
        return ok;
    };
    // group g (0-3) of the refine MMAs of the pair whose first output row is y, into buffer d:
    // [W0; W1] x row y (initialises both rows), W0 x row y-1, [W1; W2] x row y+1, W2 x row y+2
    auto refine_group = [&](uint32_t d, int y, int g) {
        const int row = g == 0 ? y : g == 1 ? y - 1 : g == 2 ? y + 1 : y + 2;
        const int ky = g < 2 ? 0 : g - 1;
        const bool n128 = g != 1 && g != 3;
        const uint32_t dd = g == 1 ? d + 64 : d;
        const uint32_t a = ring0 + slot_of(row) * SLOT;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx)
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
                mma_f16(dd, sdesc(a + 2 * kk * LBO + kx * 16, LBO, 128),
                        sdesc(b0 + ((kx * 4 + 2 * kk) * 3 + ky) * WBLK, WLBO, 128), n128 ? idesc128 : idesc64,
                        !(g == 0 && kx == 0 && kk == 0));
    };
    // half s of the current row (hs: the row's first half) into its buffer
    auto head_mma = [&](int s) {
        const int tile = s >> 1, h = s & 1, buf = (hs + s) % 3;
        const uint64_t a = sdesc(a2addr + tile * kHeadTile, kM * 16, 128);
        const uint32_t d = hcol + 64 * buf, bo = hb0 + 64 * 16 * h, id = h ? idesc_m128(48) : idesc64;
        mma_f16(d, a, sdesc(bo, 128 * 16, 128), id, 0);
        mma_f16(d, a, sdesc(bo + kHeadBCH, 128 * 16, 128), id, 1);
        mma_f16(d, sdesc(o0, kM * 16, 128), sdesc(bo + 2 * kHeadBCH, 128 * 16, 128), id, 1);
        commit(&head_full[3 * wg + buf]);
    };
    // this warp's wait for half s of the current row; false if it expired
    auto head_wait = [&](int s) {
        const int buf = (hs + s) % 3;
        const bool ok = __all_sync(0xffffffffu, mbar_wait_idle(&head_full[3 * wg + buf], (head_phase >> buf) & 1u, err,
                                                                kErrTimeout));
        if (ok) {
            head_phase ^= 1u << buf;
            fence_after_sync();
        }
        return ok;
    };
    auto head_cols = [&](int s) { return hcol + lrow + 64 * uint32_t((hs + s) % 3); };

    for (long long item = blockIdx.x; item < items && live; item += gridDim.x) {
        last_item(item, items);
        const FusedItem fi = fused_item(item, rs, nstrip, nband, band);
        if (fi.skip) continue;   // uniform across the CTA
        const int4 reg = rs.regions[fi.r];
        const int x = fi.x0 + tq;
        const bool xin = tq < kConvStrip && x < fi.px1;
        const int row0 = 2 * fi.y0 - 2;   // LR row of source ring slot 0
        const uint8_t* sfu8 = static_cast<const uint8_t*>(src.ptr) + size_t(reg.x) * plane * 3;
        const float* sff = static_cast<const float*>(src.ptr) + size_t(reg.x) * plane * 3;
        auto fetch = [&](int row, int c) -> uint3 {
            const int sy = clampi(reg.y + clampi(row, 0, rs.rh - 1) - src.pad_y, 0, src.H - 1);
            const int sx = clampi(reg.z + clampi(2 * fi.x0 - 2 + c, 0, rs.rw - 1) - src.pad_x, 0, src.W - 1);
            if (SRC_U8) {
                const uint8_t* q = sfu8 + (size_t(sy) * src.W + sx) * 3;
                return make_uint3(q[0], q[1], q[2]);
            }
            const float* q = sff + size_t(sy) * src.W + sx;
            return make_uint3(__float_as_uint(q[0]), __float_as_uint(q[plane]), __float_as_uint(q[2 * plane]));
        };
        auto put = [&](int row, int c, uint3 raw) {
            float* ps = s_src + ((row - row0) % kSrcRing) * ROWF;
            float v[3];
            if (SRC_U8) {
                v[0] = s_lut[raw.x]; v[1] = s_lut[raw.y]; v[2] = s_lut[raw.z];
            } else {
                v[0] = __uint_as_float(raw.x); v[1] = __uint_as_float(raw.y); v[2] = __uint_as_float(raw.z);
            }
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                ps[ch * 2 * kSrcArr + c] = v[ch];
                if (c > 0) ps[ch * 2 * kSrcArr + kSrcArr + c - 1] = v[ch];
            }
        };
        // both warpgroups are done with the previous item (its source rows, its MMAs observed)
        if (epilogues_sync_or(bad || dead || pbad)) {
            live = false;
            break;
        }
        // item prologue: dec540 rows y0-1 .. y0+4 and the refine MMAs of the first pair
        if (issuer) {
            bool ok = true;
            for (int row = fi.y0 - 1; row <= min(fi.y0 + 4, fi.y1); ++row) load_row(row, fi);
            for (int row = fi.y0 - 1; row <= fi.y0 + 2 && ok; ++row) ok = wait_row(row);
            if (ok) {
                fence_after_sync();
                for (int g = 0; g < 4; ++g) refine_group(tmem, fi.y0, g);
            }
            commit(ref_full);   // also on a failed wait, so that every parity stays in step
            pbad = !ok;
        }
        __syncwarp();
        for (int e = t; e < 8 * kSrcCols; e += kFusedThreads)
            put(row0 + e / kSrcCols, e % kSrcCols, fetch(row0 + e / kSrcCols, e % kSrcCols));
        for (int y0 = fi.y0; y0 < fi.y1; y0 += 2, ++p) {
            const int y = y0 + wg;
            const bool more = y0 + 2 < fi.y1;      // the item has a next pair
            const int nrow = 2 * y0 + 6;           // the next pair's first new LR source row
            // uint8 samples are held packed, one register per pixel, until the end of the pair
            uint3 pre[5];
            if (more) {
#pragma unroll
                for (int m = 0; m < 5; ++m) {
                    const int e = t + kFusedThreads * m;
                    if (e < 4 * kSrcCols) {
                        pre[m] = fetch(nrow + e / kSrcCols, e % kSrcCols);
                        if (SRC_U8) pre[m].x = pre[m].x | (pre[m].y << 8) | (pre[m].z << 16);
                    }
                }
            }
            // the source rows stored so far are visible; both warpgroups are done with the
            // previous pair
            if (epilogues_sync_or(bad || dead || pbad)) {
                live = false;
                break;
            }
            const uint32_t col = tmem + lrow + half;
            // refine epilogue -> tail operand of this row
            bad = !__all_sync(0xffffffffu, mbar_wait_idle(ref_full, p & 1, err, kErrTimeout));
            if (!bad) {
                fence_after_sync();
                // this pair's MMAs have completed: its first two dec540 slots take the rows of the
                // pair after next
                if (issuer && y0 + 4 < fi.y1) {
                    load_row(y0 + 5, fi);
                    if (y0 + 6 <= fi.y1) load_row(y0 + 6, fi);
                }
                __syncwarp();
                float vr[2][32];
                tmem_ld32x2(col, col + 32, vr[0], vr[1]);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    epi_add_leaky(vr[h], s_rb + h * 32, slope);
                    uint4 q[4];
                    pack_f16x32(vr[h], q);
#pragma unroll
                    for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(a2 + ((h * 4 + c) * kM + tq) * 16) = q[c];
                }
                fence_async_smem();
            }
            fence_before_sync();
            dead = warpgroup_sync_or(wg, bad || pbad);
            if (!dead && tq == 0) {
                fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f16(tmem + half, sdesc(a2addr + kk * 2 * kM * 16, kM * 16, 128),
                            sdesc(t0 + kk * 2 * 64 * 16, 64 * 16, 128), idesc64, kk > 0);
                commit(&tail_full[wg]);
            }
            __syncwarp();
            // tail epilogue: coefficients (tail bias, coefficient_clamp, f16) into the head's four
            // A tiles, which take the place of the tail operand (its MMAs have completed)
            if (!dead) {
                bad = !__all_sync(0xffffffffu, mbar_wait_idle(&tail_full[wg], tail_phase, err, kErrTimeout));
                if (!bad) {
                    tail_phase ^= 1u;
                    fence_after_sync();
                    float vt[2][32];
                    tmem_ld32x2(col, col + 32, vt[0], vt[1]);
                    fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(pair_empty);   // this warp's part of the pair buffer is read
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float (&v)[32] = vt[h];
                        epi_add(v, s_tb + h * 32);
#pragma unroll
                        for (int n = 0; n < 32; n += 2) {   // coefficient_clamp, as k_tc_refine_tail
                            const float2 soft = __ffma2_rn(make_float2(0.05f, 0.05f),
                                                           __fadd2_rn(make_float2(fminf(fabsf(v[n]), 12.f),
                                                                                  fminf(fabsf(v[n + 1]), 12.f)),
                                                                      make_float2(-2.f, -2.f)),
                                                           make_float2(2.f, 2.f));
                            v[n] = min_xorsign_abs(v[n], soft.x);
                            v[n + 1] = min_xorsign_abs(v[n + 1], soft.y);
                        }
                        uint4 q[4];
                        pack_f16x32(v, q);
                        // tile (h, j): channels h*32 + j*16 .. +16 = chunks q[2j], q[2j+1]
#pragma unroll
                        for (int j = 0; j < 2; ++j)
#pragma unroll
                            for (int c = 0; c < 2; ++c)
                                *reinterpret_cast<uint4*>(a2 + (2 * h + j) * kHeadTile + (c * kM + tq) * 16) = q[2 * j + c];
                    }
                    fence_async_smem();
                }
            }
            fence_before_sync();
            dead = warpgroup_sync_or(wg, dead || bad || pbad);
            if (!dead && tq == 0) {
                fence_after_sync();
                head_mma(0);
                head_mma(1);
                head_mma(2);
            }
            __syncwarp();
            // the source ring rows of LR rows 2y - 2 .. 2y + 3: tile (i, j) reads rows i .. i + 4
            const float* srow[6];
#pragma unroll
            for (int r6 = 0; r6 < 6; ++r6) srow[r6] = s_src + ((2 * y - 2 + r6 - row0) % kSrcRing) * ROWF;
            // reconstruction of the row's four tiles.  Per tile and half: wait for its MMAs, load
            // its weights, and once every thread of the warpgroup has them, issue the same half
            // of the next tile into the freed columns, then run its FMAs.
#pragma unroll
            for (int tile = 0; tile < 4; ++tile) {
                const int i = tile >> 1, j = tile & 1;
                const int Y = 2 * y + i, X = 2 * x + j;   // region-local LR pixel
                const float2* rows[5];
#pragma unroll
                for (int ky = 0; ky < 5; ++ky) rows[ky] = reinterpret_cast<const float2*>(srow[i + ky] + j * kSrcArr) + tq;
                // k_tc_head's accumulation: acc[phase][ch] = (taps with even kx and the fifth
                // column | taps with odd kx), tap pairs in column order, then the fifth column
                float2 acc[4][3];
#pragma unroll
                for (int q = 0; q < 4; ++q)
#pragma unroll
                    for (int ch = 0; ch < 3; ++ch) acc[q][ch] = make_float2(0.f, 0.f);
                {   // half 0: tap pairs of rows 0-3 (columns 0-63)
                    float w[2][32];
                    if (!dead) {
                        bad = !head_wait(2 * tile);
                        if (!bad) tmem_ld32x2(head_cols(2 * tile), head_cols(2 * tile) + 32, w[0], w[1]);
                    }
                    fence_before_sync();
                    dead = warpgroup_sync_or(wg, dead || bad || pbad);
                    if (!dead) {
                        if (2 * tile + 3 < 8 && tq == 0) {
                            fence_after_sync();
                            head_mma(2 * tile + 3);
                        }
                        __syncwarp();
#pragma unroll
                        for (int pr = 0; pr < 8; ++pr) {
                            const int ky = pr >> 1, jj = pr & 1, n = pr * 8;
#pragma unroll
                            for (int ch = 0; ch < 3; ++ch) {
                                const float2 sv = rows[ky][ch * kSrcArr + jj];
#pragma unroll
                                for (int q = 0; q < 4; ++q)
                                    acc[q][ch] = __ffma2_rn(sv, make_float2(w[n >> 5][(n & 31) + 2 * q], w[n >> 5][(n & 31) + 2 * q + 1]),
                                                            acc[q][ch]);
                            }
                        }
                    }
                }
                {   // half 1: tap pairs of row 4 (columns 64-79), fifth column (80-99)
                    uint32_t w[2][32];
                    if (!dead) {
                        bad = !head_wait(2 * tile + 1);
                        if (!bad) {
                            tmem_ld_x32(head_cols(2 * tile + 1), w[0]);
                            tmem_ld_x4(head_cols(2 * tile + 1) + 32, w[1]);
                            tmem_wait_ld();
                            tmem_regs_ready(w[0]);
                            tmem_regs_ready(w[1]);
                        }
                    }
                    fence_before_sync();
                    dead = warpgroup_sync_or(wg, dead || bad || pbad);
                    if (!dead) {
                        if (tq == 0) {
                            fence_after_sync();
                            if (2 * tile + 4 < 8) head_mma(2 * tile + 4);
                        }
                        // producer: group `tile` of the next pair's refine MMAs, behind the head
                        // MMAs; the first once both warpgroups have read this pair's tails
                        if (issuer && more) {
                            bool ok = true;
                            if (tile == 0) ok = mbar_wait_bounded(pair_empty, p & 1, err, kErrTimeout);
                            if (tile == 2) ok = wait_row(y0 + 3);
                            if (tile == 3) ok = wait_row(y0 + 4);
                            if (ok) {
                                fence_after_sync();
                                refine_group(tmem, y0 + 2, tile);
                            }
                            if (tile == 3) commit(ref_full);
                            pbad = pbad || !ok;
                        }
                        __syncwarp();
                        auto wv = [&](int n) { return __uint_as_float(n < 96 ? w[0][n - 64] : w[1][n - 96]); };
#pragma unroll
                        for (int pr = 8; pr < 10; ++pr) {
                            const int jj = pr & 1, n = pr * 8;
#pragma unroll
                            for (int ch = 0; ch < 3; ++ch) {
                                const float2 sv = rows[4][ch * kSrcArr + jj];
#pragma unroll
                                for (int q = 0; q < 4; ++q)
                                    acc[q][ch] = __ffma2_rn(sv, make_float2(wv(n + 2 * q), wv(n + 2 * q + 1)), acc[q][ch]);
                            }
                        }
#pragma unroll
                        for (int ky = 0; ky < 5; ++ky)
#pragma unroll
                            for (int ch = 0; ch < 3; ++ch) {
                                const float sv = rows[ky][ch * kSrcArr + 2].x;
#pragma unroll
                                for (int q = 0; q < 4; ++q) acc[q][ch].x = fmaf(sv, wv(80 + ky * 4 + q), acc[q][ch].x);
                            }
                    }
                }
                if (!dead && xin && Y >= fi.core.x && Y < fi.core.z && X >= fi.core.y && X < fi.core.w) {
                    float out[4][3];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
#pragma unroll
                        for (int ch = 0; ch < 3; ++ch) out[q][ch] = acc[q][ch].x + acc[q][ch].y;
                    if (!SRC_U8) {   // only float sources can make a non-finite value (k_tc_head)
                        float2 all = __fadd2_rn(make_float2(out[0][0], out[0][1]), make_float2(out[0][2], out[1][0]));
                        all = __fadd2_rn(all, __fadd2_rn(make_float2(out[1][1], out[1][2]), make_float2(out[2][0], out[2][1])));
                        all = __fadd2_rn(all, __fadd2_rn(make_float2(out[2][2], out[3][0]), make_float2(out[3][1], out[3][2])));
                        if (!isfinite(all.x + all.y)) atomicOr(nonfinite, 1);
                    }
                    const int oy = 2 * (reg.y + Y - dst.pad_y), ox = 2 * (reg.z + X - dst.pad_x);
#pragma unroll
                    for (int ii = 0; ii < 2; ++ii) {
                        if (!DST_U8) {
                            float* o = static_cast<float*>(dst.ptr) + (size_t(reg.x) * 3 * dst.OH + oy + ii) * dst.OW + ox;
                            const size_t chs = size_t(dst.OH) * dst.OW;
#pragma unroll
                            for (int ch = 0; ch < 3; ++ch)
                                *reinterpret_cast<float2*>(o + ch * chs) = make_float2(out[2 * ii][ch], out[2 * ii + 1][ch]);
                        } else {
                            const uint2 q01 = u8_code_bits2(out[2 * ii][0], out[2 * ii][1]);
                            const uint2 q23 = u8_code_bits2(out[2 * ii][2], out[2 * ii + 1][0]);
                            const uint2 q45 = u8_code_bits2(out[2 * ii + 1][1], out[2 * ii + 1][2]);
                            unsigned short* o = reinterpret_cast<unsigned short*>(
                                static_cast<uint8_t*>(dst.ptr) + ((size_t(reg.x) * dst.OH + oy + ii) * dst.OW + ox) * 3);
                            __stcs(o, (unsigned short)__byte_perm(q01.x, q01.y, 0x0040));
                            __stcs(o + 1, (unsigned short)__byte_perm(q23.x, q23.y, 0x0040));
                            __stcs(o + 2, (unsigned short)__byte_perm(q45.x, q45.y, 0x0040));
                        }
                    }
                }
            }
            hs = (hs + 8) % 3;
            // the next pair's new source rows into the slots the previous pair used
            if (more && !dead) {
#pragma unroll
                for (int m = 0; m < 5; ++m) {
                    const int e = t + kFusedThreads * m;
                    if (e < 4 * kSrcCols) {
                        if (SRC_U8) pre[m] = make_uint3(pre[m].x & 255u, (pre[m].x >> 8) & 255u, pre[m].x >> 16);
                        put(nrow + e / kSrcCols, e % kSrcCols, pre[m]);
                    }
                }
            }
        }
    }
    // every MMA this warpgroup's issuing thread committed, and every dec540 load, lands before
    // TMEM and shared memory are released (a commit covers all of the thread's earlier MMAs)
    if (tq == 0) {
        commit(&drain[wg]);
        mbar_wait_bounded(&drain[wg], 0, err, kErrTimeout, 200000000LL);
        if (issuer)
            for (int sl = 0; sl < kFusedRing; ++sl)
                if (ring_pend & (1u << sl)) mbar_wait_bounded(&ring_full[sl], (ring_phase >> sl) & 1u, err, kErrTimeout, 200000000LL);
    }
    cta_teardown(tmem, 512);
}

// Per-call host work is part of a frame's latency: device properties and kernel attributes are
// looked up or set once per device.
int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    AEISU_CUDA(cudaGetDevice(&dev));
    int n = (dev >= 0 && dev < 64) ? cache[dev].load(std::memory_order_relaxed) : 0;
    if (n == 0) {
        AEISU_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

unsigned grid_for(long long tiles, int per_sm, int sms) {
    const long long cap = (long long)sms * per_sm;
    return unsigned(tiles < cap ? (tiles > 0 ? tiles : 1) : cap);
}

template <typename K>
void smem_attr(K kernel, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;   // (kernel, device) -> bytes set
    int dev = 0;
    AEISU_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    int& have = done[{reinterpret_cast<const void*>(kernel), dev}];
    if (have >= bytes) return;
    AEISU_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    have = bytes;
}

// Programmatic stream serialisation for small calls: a kernel's CTAs may then start while the
// previous kernel of the stream finishes its last work items; each loads its weights and takes
// its TMEM, then waits for the previous kernel (cta_setup) before it reads any activation.  It
// shortens a single frame's latency by the launch and set-up of every kernel, but costs
// throughput on large batches (measured), so it is used up to a few frames' worth of pixels.
bool use_pdl(const RegionSet& rs) { return (long long)rs.R * rs.rh * rs.rw <= (8ll << 20); }

template <typename... KArgs, typename... Args>
void launch(bool pdl, void (*kernel)(KArgs...), unsigned grid, unsigned block, int smem, cudaStream_t s,
            Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = size_t(smem);
    cfg.stream = s;
    // programmatic serialisation only on created streams, not on the legacy default stream
    const bool legacy = s == nullptr || s == cudaStreamLegacy;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (pdl && !legacy) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    AEISU_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// Rows per work item: enough items to fill every CTA slot, at most 32 rows.
int pick_band(long long strips_x_regions, int rows, int slots) {
    const long long per_slot = (strips_x_regions * rows + slots - 1) / slots;
    return int(std::max<long long>(4, std::min<long long>(32, per_slot)));
}

// Rows per head work item: the band that minimises the rows the busiest CTA slot runs
// (items are dealt round-robin), counting about four rows of set-up per item.
int pick_band_balanced(long long strips_x_regions, int rows, int slots) {
    int best = 4;
    long long best_cost = -1;
    for (int band = 4; band <= std::max(4, rows); ++band) {
        const long long items = strips_x_regions * ((rows + band - 1) / band);
        const long long cost = (items + slots - 1) / slots * (band + 4);
        if (best_cost < 0 || cost < best_cost) { best = band; best_cost = cost; }
    }
    return best;
}

// Fused refine + tail + reconstruction (k_tc_refine_head): one CTA per SM, its shared memory
// request raised near the SM's limit so that no CTA of the other stream's tensor-core kernels
// shares the SM and waits there for the TMEM this kernel holds until its last item.
void launch_refine_head(const SrcDesc& src, const RegionSet& rs, const DstDesc& dst, const TcWeights& w,
                        void* dec540, const uint8_t* head_img, int* nonfinite, int* err, cudaStream_t s, bool pdl,
                        int sms) {
    if ((long long)rs.R * rs.core_h * rs.core_w == 0) return;
    const int ph = rs.rh / 2, pw = rs.rw / 2;
    // packed columns and rows a core can cover (its rows rounded out to whole pairs)
    const int nstrip = (rs.core_w / 2 + 1 + kConvStrip - 1) / kConvStrip;
    const int span = std::min(ph, rs.core_h / 2 + 3);
    // even band minimising the rows of the busiest CTA, counting about six rows of set-up per item
    int band = 2;
    long long best = -1;
    for (int b = 2; b <= span + 1; b += 2) {
        const long long items = (long long)rs.R * nstrip * ((span + b - 1) / b);
        const long long cost = (items + sms - 1) / sms * (b + 6);
        if (best < 0 || cost < best) { best = cost; band = b; }
    }
    const int nband = (span + band - 1) / band;
    const long long items = (long long)rs.R * nstrip * nband;
    const CUtensorMap map = make_row_window_map(dec540, rs.R, ph, 4, pw, kM);
    auto k = src.kind == 0 ? (dst.kind == 0 ? k_tc_refine_head<true, true> : k_tc_refine_head<true, false>)
                           : (dst.kind == 0 ? k_tc_refine_head<false, true> : k_tc_refine_head<false, false>);
    constexpr int bytes = 220 * 1024;
    static_assert(bytes >= kFusedBytes, "fused kernel's shared memory");
    smem_attr(k, bytes);
    launch(pdl, k, grid_for(items, 1, sms), kFusedThreads, bytes, s, map, rs, w.refine, w.tail, w.refine_bias,
           w.tail_bias, w.slope, head_img, src, dst, band, nstrip, nband, nonfinite, err);
}

}  // namespace

void launch_tc_controller(int route, const SrcDesc& src, const RegionSet& rs, const TcWeights& w, void* enc540,
                          void* encu, void* low_a, void* low_b, void* dec540, void* meta, float* raw_meta,
                          int* err, cudaStream_t s, int* launches, const StageMark& mark, const FusedHead* head) {
    const int sms = sm_count();
    const bool pdl = use_pdl(rs);
    const bool fp8 = route == kRouteE4M3, i8 = route == kRouteI8;
    const int ph = rs.rh / 2, pw = rs.rw / 2, lh = rs.rh / 4, lw = rs.rw / 4;
    const long long low_tiles = (long long)rs.R * lh * ((lw + kM - 1) / kM);
    {
        const long long strips = (long long)rs.R * ((pw + kM - 1) / kM);
        const int band = pick_band(strips, ph, sms * 5);
        const long long items = strips * ((ph + band - 1) / band);
        const int bytes = 2 * 4 * kM * 16 + 4 * 32 * 16 + kProjRing * kProjTW * 16;   // five CTAs per SM
        auto kp = src.kind == 0 ? (fp8 ? k_tc_project<true, false, true> : i8 ? k_tc_project<false, true, true> : k_tc_project<false, false, true>)
                                : (fp8 ? k_tc_project<true, false, false> : i8 ? k_tc_project<false, true, false> : k_tc_project<false, false, false>);
        smem_attr(kp, bytes);
        launch(pdl, kp, grid_for(items, 5, sms), kThreads, bytes, s, src, rs, w.proj, w.project, w.slope, w.inv_s1, enc540, encu, band, err);
    }
    mark(1);
    {
        const int kch = fp8 ? 8 : 16;
        const int bytes = kch * kM * 16 + kch * 64 * 16;
        auto kc = fp8 ? k_tc_compress<true> : i8 ? k_tc_compress<false, true> : k_tc_compress<false>;
        smem_attr(kc, bytes);
        launch(pdl, kc, grid_for(low_tiles, 4, sms), kThreads, bytes, s, rs, w.compress, w.compress_ep, w.compress_cp, encu, low_a, err);
    }
    {
        // one group per CTA (two CTAs per work item), four CTAs per SM; bands hold whole row pairs
        const int ich = fp8 ? 4 : 8, cpg = ich / 2;
        const int bytes = 1024 + kRing * cpg * kM * 16 + 9 * cpg * 32 * 16;
        const int slots = sms * 2;   // work items in flight: two CTAs each
        const long long strips = (long long)rs.R * ((lw + kConvStrip - 1) / kConvStrip);
        const int band = (pick_band(strips, lh, slots) + 1) & ~1;   // lh is a multiple of 8
        const long long items = strips * ((lh + band - 1) / band);
        const unsigned grid = 2 * grid_for(items, 2, sms);
        const CUtensorMap map_a = make_row_window_map(low_a, rs.R, lh, ich, lw, kM, cpg);
        const CUtensorMap map_b = make_row_window_map(low_b, rs.R, lh, ich, lw, kM, cpg);
        void* bufs[2] = {low_a, low_b};
        const CUtensorMap* maps[2] = {&map_a, &map_b};
        auto kk = fp8 ? k_tc_core<true> : i8 ? k_tc_core<false, true> : k_tc_core<false>;
        smem_attr(kk, bytes);
        for (int i = 0; i < 4; ++i)
            launch(pdl, kk, grid, kWsThreads, bytes, s, *maps[i & 1], rs, w.core[i], w.core_ep[i], w.core_cp[i], bufs[(i + 1) & 1], band, err);
    }
    mark(2);
    {
        const int kch = fp8 ? 4 : 8;
        const int bytes = kch * kM * 16 + kch * 128 * 16;
        auto ke = fp8 ? k_tc_expand<true> : i8 ? k_tc_expand<false, true> : k_tc_expand<false>;
        smem_attr(ke, bytes);
        launch(pdl, ke, grid_for(low_tiles, 4, sms), kThreads, bytes, s, rs, w.expand, w.expand_ep, w.expand_cp, low_a, enc540, dec540, err);
    }
    mark(3);
    if (head) {
        launch_refine_head(src, rs, *head->dst, w, dec540, head->head_img, head->nonfinite, err, s, pdl, sms);
    } else {
        const int bytes = 1024 + kRing * 4 * kM * 16 + 36 * 64 * 16 + 8 * 64 * 16 + 2 * 8 * kM * 16;
        const long long strips = (long long)rs.R * ((pw + kConvStrip - 1) / kConvStrip);
        const int span = refine_span(rs, raw_meta == nullptr);
        const int band = (pick_band(strips, span, sms * 2) + 1) & ~1;   // whole row pairs (ph is even)
        const long long items = strips * ((span + band - 1) / band);
        const CUtensorMap map = make_row_window_map(dec540, rs.R, ph, 4, pw, kM);
        smem_attr(k_tc_refine_tail, bytes);
        launch(pdl, k_tc_refine_tail, grid_for(items, 2, sms), kRefineThreads, bytes, s, map, rs, w.refine, w.tail, w.rbias, w.slope, meta, raw_meta, band, err);
    }
    AEISU_CUDA(cudaGetLastError());
    *launches += 8;
    mark(4);
}

namespace {

template <int PX>
void launch_tc_head_px(const SrcDesc& src, const RegionSet& rs, const DstDesc& dst, const CUtensorMap& map,
                       const uint8_t* head_img, int* nonfinite, int* err, cudaStream_t s) {
    const int sms = sm_count();
    const bool pdl = use_pdl(rs);
    constexpr int per_sm = PX == 1 ? 4 : 2;
    const long long strips = (long long)rs.R * ((rs.core_w + head_strip(PX) - 1) / head_strip(PX));
    const int band = pick_band_balanced(strips, rs.core_h, sms * per_sm);
    const long long items = strips * ((rs.core_h + band - 1) / band);
    auto k = src.kind == 0 ? (dst.kind == 0 ? k_tc_head<PX, true, true> : k_tc_head<PX, true, false>)
                           : (dst.kind == 0 ? k_tc_head<PX, false, true> : k_tc_head<PX, false, false>);
    smem_attr(k, head_smem(PX));
    launch(pdl, k, grid_for(items, per_sm, sms), kThreads, head_smem(PX), s, map, src, rs, dst, head_img, band,
           nonfinite, err);
}

}  // namespace

void launch_tc_head(const SrcDesc& src, const RegionSet& rs, const DstDesc& dst, const void* meta,
                    const uint8_t* head_img, int* nonfinite, int* err, cudaStream_t s, int* launches) {
    if ((long long)rs.R * rs.core_h * rs.core_w == 0) return;
    // coefficient rows: the chunk-planar [R][rh][2][rw][16 B] tensor, one box = 128 pixels x 2 chunks
    const CUtensorMap map = make_row_window_map(meta, rs.R, rs.rh, 2, rs.rw, kM);
    // one pixel per thread: four CTAs of 128 TMEM columns per SM (16 warps) hide the per-row MMA
    // and barrier waits better than two pixels per thread at two CTAs of 256 columns, which
    // measured 2.4% slower on 64 x 720p despite 15% fewer instructions per pixel
    launch_tc_head_px<1>(src, rs, dst, map, head_img, nonfinite, err, s);
    AEISU_CUDA(cudaGetLastError());
    *launches += 1;
}

}  // namespace aeisu
