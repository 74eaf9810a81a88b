// Training-time reconstruction: reconstruct() of aeisu/reconstruction.py:29-83 as a standalone
// operator on caller-given metadata, base and basis (FP32), and its backward, which the
// reference leaves to autograd (train.py:99-103).  Paths are relative to the AELabs42/AEISU
// checkout.
//
//   k_recon_fwd       one thread per core LR pixel, persistent CTAs over 4 x 64 pixel tiles.
//                     The 5x5 RGB window of the tile sits in shared memory, the 1,700-float bank
//                     (base [25][4], basis [25][16][4]) in constant memory.  Per tap the four
//                     phase weights are base + sum_k c_k basis[tap][k] (the reference's einsum
//                     then base add), applied to the three channels (phase pairs as packed
//                     f32x2 FMAs).
//   k_recon_bwd       same tiles, the basis in constant memory.  Per pixel and tap, the filter gradient
//                     gw[p] = sum_c grad[c][p] src[c][tap]; the coefficient gradient
//                     gc[k] = sum_{tap,p} gw[p] basis[tap][k][p], through the clamp's derivative
//                     (1 where |v| <= 2, 0.05 on the soft ramp up to 2.5 inclusive, else 0) into
//                     the metadata layout.  Pixels the gradient sample selects (all of them at
//                     stride 1, one in stride^2 otherwise) leave their gw and s^2 * c_k in a
//                     shared-memory slot list in thread order; after each tile the CTA adds
//                     their outer products into per-thread accumulators of the 17 x 100
//                     base/basis gradient.  Each CTA writes its partial once.
//                     With trim > 0 it first zeroes the metadata gradients of the pixels
//                     outside the core, which the reference's crop gives no gradient.
//   k_recon_reduce    sums the partials of all CTAs in a fixed order (deterministic for a given
//                     grid), writing grad_base [25][4] and grad_basis [25][16][4].
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <mutex>
#include <utility>

#include "common.h"
#include "kernels.h"

namespace aeisu {
namespace {

constexpr int kRTX = 64, kRTY = 4;          // tile: 4 core rows x 64 core columns, one pixel per thread
constexpr int kRThreads = kRTX * kRTY;
constexpr int kRWinX = kRTX + 4, kRWinY = kRTY + 4;
constexpr int kBase = 25 * 4;               // bank floats: base [25][4], then basis [25][16][4]
constexpr int kBank = kBase + 25 * 16 * 4;
constexpr int kGrad = 17 * 100;             // base/basis gradient: [k 0..15 | 16 = base][tap * 4 + phase]
constexpr int kRedThreads = 200;            // threads owning gradient outputs: tp = t % 100, k half = t / 100
constexpr int kSlotW = 100;                 // floats of one slot's filter gradient
constexpr int kSlotC = 20;                  // floats of one slot's s^2 * c_k (17 used, 16-byte rows)

struct ReconJob {
    const float* src;      // [n][3][h][w]
    const float* meta;     // [n][64][h/2][w/2]
    const float* base;     // [25][4]
    const float* basis;    // [25][16][4]
    const float* grad;     // [n][3][2ch][2cw] (backward)
    float* out;            // [n][3][2ch][2cw] (forward)
    float* gmeta;          // [n][64][h/2][w/2] (backward)
    float* partial;        // [grid][kGrad] (backward, stride > 0)
    int n, h, w, off, ch, cw;
    int stride, phase;     // phase already reduced mod stride^2
    int tiles_x, tiles_y;
    long long tiles;
    int slots;             // slot capacity per tile (0 when stride == 0)
};

// The bank is the same for every thread, so it sits in constant memory, where a packed f32x2
// FMA reads a pair of it as a direct operand: no load instruction and no shared-memory
// wavefront per FMA (a broadcast 16-byte shared load costs two wavefronts; with the bank in
// shared memory they bound both kernels).  Scalar FMAs on constant operands were slower still
// in the backward (0.46 ms per training step against 0.37 from shared memory and 0.31 with
// pairs): one issue slot per FMA.  Each call copies its base/basis here on its own stream,
// after the previous call of its kind has finished with them (see reconstruct_f32).
__constant__ float c_fwd_bank[kBank];   // base [25][4], then basis [25][16][4]
__constant__ float c_bwd_basis[kBank - kBase];   // backward: basis [25][16][4]

__device__ __forceinline__ float clamp_coef(float v) {
    // reconstruction.py:15-17 with the reference's own operations and comparisons
    const float mag = fabsf(v);
    if (mag <= 2.f) return v;
    const float soft = fminf(__fadd_rn(2.f, __fmul_rn(0.05f, __fsub_rn(mag, 2.f))), 2.5f);
    return v > 0.f ? soft : (v < 0.f ? -soft : __fmul_rn(v, soft));   // sign(v) * soft (NaN stays NaN)
}

__device__ __forceinline__ float clamp_grad(float v, float g) {
    const float mag = fabsf(v);
    if (mag <= 2.f) return g;
    const float soft = __fadd_rn(2.f, __fmul_rn(0.05f, __fsub_rn(mag, 2.f)));
    return soft <= 2.5f ? __fmul_rn(0.05f, g) : 0.f;
}

// Stage the bank and the tile's source window (rows y0-2 .. y0+TY+1, columns x0-2 .. x0+TX+1 of
// the core, clamped into the frame: replicate padding at trim 0, the real border otherwise).
__device__ __forceinline__ void stage_window(const ReconJob& j, int b, int y0, int x0, float (*win)[kRWinY][kRWinX]) {
    const size_t plane = size_t(j.h) * j.w;
    const float* s = j.src + size_t(b) * 3 * plane;
    for (int i = threadIdx.x; i < 3 * kRWinY * kRWinX; i += kRThreads) {
        const int c = i / (kRWinY * kRWinX), r = (i / kRWinX) % kRWinY, x = i % kRWinX;
        const int Y = min(max(j.off + y0 - 2 + r, 0), j.h - 1);
        const int X = min(max(j.off + x0 - 2 + x, 0), j.w - 1);
        win[c][r][x] = __ldg(s + c * plane + size_t(Y) * j.w + X);
    }
}

__device__ __forceinline__ void tile_origin(const ReconJob& j, long long tile, int& b, int& y0, int& x0) {
    const long long per = (long long)j.tiles_x * j.tiles_y;
    b = int(tile / per);
    const int r = int(tile % per);
    y0 = (r / j.tiles_x) * kRTY;
    x0 = (r % j.tiles_x) * kRTX;
}

// Metadata offset of core pixel (y, x): channel parity * 16 (+ k * plane), parity = 2 (Y&1) + (X&1).
__device__ __forceinline__ size_t meta_at(const ReconJob& j, int b, int y, int x) {
    const int Y = j.off + y, X = j.off + x, hh = j.h >> 1, ww = j.w >> 1;
    const int parity = 2 * (Y & 1) + (X & 1);
    return ((size_t(b) * 64 + parity * 16) * hh + (Y >> 1)) * ww + (X >> 1);
}

__global__ void __launch_bounds__(kRThreads) k_recon_fwd(ReconJob j) {
    __shared__ float s_win[3][kRWinY][kRWinX];
    const int tx = threadIdx.x % kRTX, ty = threadIdx.x / kRTX;
    const size_t kplane = size_t(j.h >> 1) * (j.w >> 1);
    const int OH = 2 * j.ch, OW = 2 * j.cw;
    for (long long tile = blockIdx.x; tile < j.tiles; tile += gridDim.x) {
        int b, y0, x0;
        tile_origin(j, tile, b, y0, x0);
        __syncthreads();   // the previous tile's window is no longer read
        stage_window(j, b, y0, x0, s_win);
        __syncthreads();
        const int y = y0 + ty, x = x0 + tx;
        if (y >= j.ch || x >= j.cw) continue;
        float2 cc[16];   // (c, c): one coefficient for both lanes of a phase pair
        const float* mp = j.meta + meta_at(j, b, y, x);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float c = clamp_coef(__ldg(mp + k * kplane));
            cc[k] = make_float2(c, c);
        }
        float2 o01[3], o23[3];   // phases (0, 1) and (2, 3) per channel
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) o01[ch] = o23[ch] = make_float2(0.f, 0.f);
#pragma unroll
        for (int t = 0; t < 25; ++t) {   // every bank index is a compile-time constant
            const int ky = t / 5, kx = t % 5;
            float2 w01 = make_float2(0.f, 0.f), w23 = w01;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float* bk = c_fwd_bank + kBase + (t * 16 + k) * 4;
                w01 = __ffma2_rn(cc[k], make_float2(bk[0], bk[1]), w01);
                w23 = __ffma2_rn(cc[k], make_float2(bk[2], bk[3]), w23);
            }
            // the reference's einsum, then the base add (reconstruction.py:70)
            const float2 a = __fadd2_rn(make_float2(c_fwd_bank[t * 4 + 0], c_fwd_bank[t * 4 + 1]), w01);
            const float2 d = __fadd2_rn(make_float2(c_fwd_bank[t * 4 + 2], c_fwd_bank[t * 4 + 3]), w23);
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                const float sv = s_win[ch][ty + ky][tx + kx];
                o01[ch] = __ffma2_rn(make_float2(sv, sv), a, o01[ch]);
                o23[ch] = __ffma2_rn(make_float2(sv, sv), d, o23[ch]);
            }
        }
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            float* op = j.out + ((size_t(b) * 3 + ch) * OH + 2 * y) * OW + 2 * x;
            *reinterpret_cast<float2*>(op) = o01[ch];        // HR row 2y: phases 0, 1
            *reinterpret_cast<float2*>(op + OW) = o23[ch];   // HR row 2y + 1: phases 2, 3
        }
    }
}

// trim > 0: metadata gradients of pixels outside the core are zero (the reference's crop gives
// them none).  A grid-stride pass over the metadata positions of the border, one thread per
// (frame, parity, position), before the CTA's tiles.
__device__ __forceinline__ void zero_border(const ReconJob& j) {
    const int hh = j.h >> 1, ww = j.w >> 1;
    const long long total = (long long)j.n * 4 * hh * ww;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int xx = int(i % ww), yy = int((i / ww) % hh), parity = int((i / ((long long)ww * hh)) % 4);
        const int b = int(i / (4LL * ww * hh));
        const int Y = 2 * yy + (parity >> 1), X = 2 * xx + (parity & 1);
        if (Y >= j.off && Y < j.off + j.ch && X >= j.off && X < j.off + j.cw) continue;
        float* g = j.gmeta + ((size_t(b) * 64 + parity * 16) * hh + yy) * ww + xx;
#pragma unroll
        for (int k = 0; k < 16; ++k) g[size_t(k) * hh * ww] = 0.f;
    }
}

__global__ void __launch_bounds__(kRThreads, 2) k_recon_bwd(ReconJob j) {
    __shared__ float s_win[3][kRWinY][kRWinX];
    __shared__ int s_wsel[kRThreads / 32];
    extern __shared__ __align__(16) float s_dyn[];
    float* s_gw = s_dyn;                                   // [slots][100]
    float* s_mc = s_dyn + size_t(j.slots) * kSlotW;        // [slots][20]
    if (j.off > 0) zero_border(j);
    const int tx = threadIdx.x % kRTX, ty = threadIdx.x / kRTX;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t kplane = size_t(j.h >> 1) * (j.w >> 1);
    const int OH = 2 * j.ch, OW = 2 * j.cw;
    const int s = j.stride;
    const float m = float(s) * float(s);   // stride 1: weight 1
    // base/basis gradient accumulators of this thread: tp = t % 100, k = kh*9 .. (kh ? 16 : 8)
    const bool red = s > 0 && threadIdx.x < kRedThreads;
    const int tp = threadIdx.x % 100, kh = threadIdx.x / 100;
    float acc[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) acc[i] = 0.f;
    for (long long tile = blockIdx.x; tile < j.tiles; tile += gridDim.x) {
        int b, y0, x0;
        tile_origin(j, tile, b, y0, x0);
        const int y = y0 + ty, x = x0 + tx;
        const bool core = y < j.ch && x < j.cw;
        const bool sel = core && s > 0 && (s == 1 || (y % s == j.phase / s && x % s == j.phase % s));
        const unsigned ball = __ballot_sync(0xffffffffu, sel);
        __syncthreads();   // the previous tile's window and slots are no longer read
        if (lane == 0) s_wsel[warp] = __popc(ball);
        stage_window(j, b, y0, x0, s_win);
        __syncthreads();
        int slot = -1, nsel = 0;
        for (int w = 0; w < kRThreads / 32; ++w) {
            if (w < warp) slot += s_wsel[w];
            nsel += s_wsel[w];
        }
        slot = sel ? slot + 1 + __popc(ball & ((1u << lane) - 1u)) : -1;
        if (core) {
            const size_t mo = meta_at(j, b, y, x);
            float2 g01[3], g23[3];
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const float* gp = j.grad + ((size_t(b) * 3 + c) * OH + 2 * y) * OW + 2 * x;
                g01[c] = __ldg(reinterpret_cast<const float2*>(gp));
                g23[c] = __ldg(reinterpret_cast<const float2*>(gp + OW));
            }
            float2 gc[16];   // (phases 0 + 2, phases 1 + 3) partial sums of each coefficient gradient
#pragma unroll
            for (int k = 0; k < 16; ++k) gc[k] = make_float2(0.f, 0.f);
            float* gw_slot = slot >= 0 ? s_gw + size_t(slot) * kSlotW : nullptr;
#pragma unroll
            for (int t = 0; t < 25; ++t) {   // every bank index is a compile-time constant
                const int ky = t / 5, kx = t % 5;
                float2 w01 = make_float2(0.f, 0.f), w23 = w01;
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    const float sv = s_win[c][ty + ky][tx + kx];
                    w01 = __ffma2_rn(make_float2(sv, sv), g01[c], w01);
                    w23 = __ffma2_rn(make_float2(sv, sv), g23[c], w23);
                }
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const float* bk = c_bwd_basis + (t * 16 + k) * 4;
                    gc[k] = __ffma2_rn(w01, make_float2(bk[0], bk[1]), gc[k]);
                    gc[k] = __ffma2_rn(w23, make_float2(bk[2], bk[3]), gc[k]);
                }
                if (gw_slot) reinterpret_cast<float4*>(gw_slot)[t] = make_float4(w01.x, w01.y, w23.x, w23.y);
            }
            // the raw coefficients are needed only now (the clamp's derivative and the slot)
            float v[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) v[k] = __ldg(j.meta + mo + k * kplane);
#pragma unroll
            for (int k = 0; k < 16; ++k)
                j.gmeta[mo + k * kplane] = clamp_grad(v[k], __fadd_rn(gc[k].x, gc[k].y));
            if (slot >= 0) {
                float* mc = s_mc + size_t(slot) * kSlotC;
#pragma unroll
                for (int k = 0; k < 16; ++k) mc[k] = __fmul_rn(m, clamp_coef(v[k]));
                mc[16] = m;
            }
        }
        if (nsel == 0) continue;   // uniform: every thread summed the same counts
        __syncthreads();           // slots written
        if (red) {
            for (int q = 0; q < nsel; ++q) {
                const float g = s_gw[size_t(q) * kSlotW + tp];
                const float* mc = s_mc + size_t(q) * kSlotC + kh * 9;
#pragma unroll
                for (int i = 0; i < 9; ++i)
                    if (kh == 0 || i < 8) acc[i] = fmaf(mc[i], g, acc[i]);
            }
        }
    }
    if (red) {
        float* p = j.partial + size_t(blockIdx.x) * kGrad;
#pragma unroll
        for (int i = 0; i < 9; ++i)
            if (kh == 0 || i < 8) p[(kh * 9 + i) * 100 + tp] = acc[i];
    }
}

// grad_base[t][p] = sum of k-row 16; grad_basis[t][k][p] = k-row k, at column t * 4 + p.  One
// block per 32 outputs: lane l owns output 32 * block + l, warp w sums the partials of CTAs
// w, w + 8, ... in order (coalesced 128-byte rows), then the eight warp sums are added in warp
// order: the same order on every call.
constexpr int kRedWarps = 8;
__global__ void __launch_bounds__(32 * kRedWarps) k_recon_reduce(const float* __restrict__ partial, int nblk,
                                                                 float* gbase, float* gbasis) {
    __shared__ float s_part[kRedWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int o = blockIdx.x * 32 + lane;
    float sum = 0.f;
    if (o < kGrad)
        for (int c = warp; c < nblk; c += kRedWarps) sum = __fadd_rn(sum, __ldg(partial + size_t(c) * kGrad + o));
    s_part[warp][lane] = sum;
    __syncthreads();
    if (warp != 0 || o >= kGrad) return;
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kRedWarps; ++w) total = __fadd_rn(total, s_part[w][lane]);
    const int k = o / 100, tpv = o % 100, t = tpv >> 2, p = tpv & 3;
    if (k == 16) gbase[tpv] = total;
    else gbasis[(t * 16 + k) * 4 + p] = total;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        AEISU_CUDA(cudaGetDevice(&prev));
        if (prev != dev) AEISU_CUDA(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
    }
};

// reconstruction.py:37-52, in the reference's order and words.
ReconJob plan_recon(int n, int h, int w, int trim, int stride, int phase) {
    require(n >= 1 && h >= 1 && w >= 1, "Expected NCHW RGB source");
    require(trim >= 0 && trim % 2 == 0 && (trim == 0 || trim >= 4),
            "trim must be zero or an even HR border of at least 4 pixels");
    require(stride >= 0 && phase >= 0, "gradient_stride and phase must be nonnegative");
    ReconJob j{};
    j.n = n;
    j.h = h;
    j.w = w;
    j.off = trim / 2;
    j.ch = h - 2 * j.off;
    j.cw = w - 2 * j.off;
    // odd h or w: the reference's reshape of the unpacked coefficients fails as well
    require(j.ch > 0 && j.cw > 0 && h % 2 == 0 && w % 2 == 0, "Source, metadata or trim geometry is invalid");
    require(stride <= 46340, "gradient_stride is too large");
    j.stride = stride;
    j.phase = stride > 1 ? int((long long)phase % ((long long)stride * stride)) : 0;
    j.tiles_x = (j.cw + kRTX - 1) / kRTX;
    j.tiles_y = (j.ch + kRTY - 1) / kRTY;
    j.tiles = (long long)n * j.tiles_x * j.tiles_y;
    // selected pixels of one tile: at most ceil(TY / s) rows x ceil(TX / s) columns
    j.slots = stride == 0 ? 0 : ((kRTY + stride - 1) / stride) * ((kRTX + stride - 1) / stride);
    return j;
}

// Per-call host work is part of a training step's latency: SM counts, occupancy-derived grids
// and the workspace pool are set up once per device (and per shared-memory size).
struct DeviceState {
    int sms = 0;
    long long fwd_ctas = 0;                 // resident k_recon_fwd CTAs
    std::map<size_t, long long> bwd_ctas;   // resident k_recon_bwd CTAs per dynamic smem size
    cudaMemPool_t pool = nullptr;           // backward partials; keeps its memory between calls
    // One constant bank of each kind per device: a call's copy waits (on its own stream) for the
    // previous call of its kind to be done with it, and calls are enqueued one at a time.
    std::mutex bank_mu;
    cudaEvent_t fwd_done = nullptr, bwd_done = nullptr;
};

std::mutex g_state_mu;
std::map<int, DeviceState> g_state;

// The largest dynamic shared memory the backward takes: every pixel of a tile selected.
constexpr size_t kMaxDyn = size_t(kRThreads) * (kSlotW + kSlotC) * sizeof(float);

DeviceState& state_of(int device) {
    std::lock_guard<std::mutex> lock(g_state_mu);
    DeviceState& d = g_state[device];
    if (d.sms == 0) {
        int sms = 0, per_sm = 0;
        AEISU_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        AEISU_CUDA(cudaFuncSetAttribute(k_recon_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMaxDyn)));
        AEISU_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_recon_fwd, kRThreads, 0));
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        AEISU_CUDA(cudaMemPoolCreate(&d.pool, &props));
        uint64_t keep = UINT64_MAX;
        AEISU_CUDA(cudaMemPoolSetAttribute(d.pool, cudaMemPoolAttrReleaseThreshold, &keep));
        AEISU_CUDA(cudaEventCreateWithFlags(&d.fwd_done, cudaEventDisableTiming));
        AEISU_CUDA(cudaEventCreateWithFlags(&d.bwd_done, cudaEventDisableTiming));
        d.fwd_ctas = (long long)std::max(per_sm, 1) * sms;
        d.sms = sms;
    }
    return d;
}

long long bwd_ctas(DeviceState& d, size_t dyn) {
    std::lock_guard<std::mutex> lock(g_state_mu);
    auto it = d.bwd_ctas.find(dyn);
    if (it != d.bwd_ctas.end()) return it->second;
    int per_sm = 0;
    AEISU_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_recon_bwd, kRThreads, dyn));
    const long long n = (long long)std::max(per_sm, 1) * d.sms;
    d.bwd_ctas.emplace(dyn, n);
    return n;
}

}  // namespace

void reconstruct_f32(const float* src, const float* meta, const float* base, const float* basis, int n, int h,
                     int w, int trim, int device, float* out, cudaStream_t stream) {
    require(src && meta && base && basis && out, "tensor pointer is null");
    ReconJob j = plan_recon(n, h, w, trim, 1, 0);
    DeviceGuard guard(device);
    j.src = src;
    j.meta = meta;
    j.base = base;
    j.basis = basis;
    j.out = out;
    DeviceState& ds = state_of(device);
    const long long grid = std::min<long long>(j.tiles, ds.fwd_ctas);
    std::lock_guard<std::mutex> lock(ds.bank_mu);
    AEISU_CUDA(cudaStreamWaitEvent(stream, ds.fwd_done, 0));   // the previous forward has read the bank
    AEISU_CUDA(cudaMemcpyToSymbolAsync(c_fwd_bank, base, kBase * sizeof(float), 0, cudaMemcpyDeviceToDevice, stream));
    AEISU_CUDA(cudaMemcpyToSymbolAsync(c_fwd_bank, basis, (kBank - kBase) * sizeof(float), kBase * sizeof(float),
                                       cudaMemcpyDeviceToDevice, stream));
    k_recon_fwd<<<unsigned(grid), kRThreads, 0, stream>>>(j);
    AEISU_CUDA(cudaGetLastError());
    AEISU_CUDA(cudaEventRecord(ds.fwd_done, stream));
}

void reconstruct_backward_f32(const float* src, const float* meta, const float* basis, const float* grad, int n,
                              int h, int w, int trim, int stride, int phase, int device, float* gmeta,
                              float* gbase, float* gbasis, cudaStream_t stream) {
    require(src && meta && basis && grad && gmeta, "tensor pointer is null");
    require(stride == 0 || (gbase && gbasis), "grad_base and grad_basis are required when gradient_stride > 0");
    ReconJob j = plan_recon(n, h, w, trim, stride, phase);
    DeviceGuard guard(device);
    j.src = src;
    j.meta = meta;
    j.basis = basis;
    j.grad = grad;
    j.gmeta = gmeta;
    const size_t dyn = size_t(j.slots) * (kSlotW + kSlotC) * sizeof(float);
    DeviceState& ds = state_of(device);
    const long long grid = std::min<long long>(j.tiles, bwd_ctas(ds, dyn));
    void* ws = nullptr;
    if (stride > 0) {
        AEISU_CUDA(cudaMallocFromPoolAsync(&ws, size_t(grid) * kGrad * sizeof(float), ds.pool, stream));
        j.partial = static_cast<float*>(ws);
    }
    cudaError_t e = cudaSuccess;
    {
        std::lock_guard<std::mutex> lock(ds.bank_mu);
        e = cudaStreamWaitEvent(stream, ds.bwd_done, 0);   // the previous backward has read the basis
        if (e == cudaSuccess)
            e = cudaMemcpyToSymbolAsync(c_bwd_basis, basis, (kBank - kBase) * sizeof(float), 0,
                                        cudaMemcpyDeviceToDevice, stream);
        if (e == cudaSuccess) {
            k_recon_bwd<<<unsigned(grid), kRThreads, dyn, stream>>>(j);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaEventRecord(ds.bwd_done, stream);
    }
    if (e == cudaSuccess && stride > 0) {
        k_recon_reduce<<<(kGrad + 31) / 32, 32 * kRedWarps, 0, stream>>>(j.partial, int(grid), gbase, gbasis);
        e = cudaGetLastError();
    }
    if (ws) cudaFreeAsync(ws, stream);
    AEISU_CUDA(e);
}

}  // namespace aeisu
