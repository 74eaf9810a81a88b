// Evaluation metrics on the GPU: encoded-Y MSE / PSNR and Gaussian-window SSIM in FP64,
// the definition of aeisu/metrics.py:11-39 (luma 11-14, distortion 17-39):
//   a = clamp(prediction, 0, 1), b = target, both cropped by `crop` pixels on every side;
//   Y = (65.481 R + 128.553 G + 24.966 B + 16) / 255 (BT.601 encoded luma) in FP64;
//   y_mse = mean (Y_a - Y_b)^2, y_psnr = -10 log10(y_mse) (inf when 0);
//   y_ssim = mean over the valid 11x11 windows (Gaussian, sigma 1.5) of
//            (2 mu_a mu_b + C1)(2 cov + C2) / ((mu_a^2 + mu_b^2 + C1)(var_a + var_b + C2)),
//   C1 = 0.01^2, C2 = 0.03^2, var and cov from the smoothed squares and product.
//
// One pass over both images, FP64-pipe bound (about 200 FP64 operations per pixel against
// 24 bytes of input).  A CTA of 128 threads owns a strip of 118 window columns and a band of
// window rows; it streams the band's input rows once: per row every thread converts one column
// of both images to Y (prefetched a row ahead), the pair goes to shared memory, and each of the
// first 118 threads takes the 11-tap horizontal Gaussian sums of Y_a, Y_b, Y_a^2, Y_b^2,
// Y_a Y_b for its window column.  Those five sums of the last 11 rows stay in registers (a
// ring unrolled by 11, so every index is static) and the vertical 11-tap sums of the ring give
// the window statistics of one output row.  The 2-D window is the outer product of the 1-D
// kernel, so the separable sums equal the reference's 2-D convolution up to FP64 rounding.
// Per-CTA partial sums (SSIM, squared error) are reduced per frame in a fixed order, so the
// result does not depend on scheduling.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <algorithm>
#include <limits>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "kernels.h"

namespace aeisu {
namespace {

constexpr int kMetThreads = 128;
constexpr int kWin = 11;
constexpr int kMetCols = kMetThreads - (kWin - 1);   // window columns per strip (118)

struct MetricJob {
    const float* pred;   // n x 3 x H x W
    const float* tgt;
    int H, W, crop;
    int Hc, Wc, Ho, Wo;  // cropped size, window grid
    int nstrip, nband, band;
    double g[kWin];      // normalised 1-D Gaussian
    double* partial;     // [items][2]: SSIM sum, squared-error sum
    int* bad;            // [n]: a non-finite input value was seen
};

__device__ __forceinline__ double luma(float r, float g, float b) {
    // ((R*65.481 + G*128.553) + B*24.966 + 16) / 255, each step rounded (no contraction), as
    // (rgb * weights).sum(dim=0) + 16 then / 255 evaluates in FP64
    double s = __dadd_rn(__dmul_rn(double(r), 65.481), __dmul_rn(double(g), 128.553));
    s = __dadd_rn(s, __dmul_rn(double(b), 24.966));
    return __ddiv_rn(__dadd_rn(s, 16.0), 255.0);
}

__device__ __forceinline__ float clamp01(float v) { return fminf(fmaxf(v, 0.f), 1.f); }

__global__ void __launch_bounds__(kMetThreads, 2) k_metric_ssim(const MetricJob j) {
    __shared__ double2 s_y[2][kMetThreads];
    const int per_frame = j.nstrip * j.nband;
    const int f = blockIdx.x / per_frame, rem = blockIdx.x % per_frame;
    const int strip = rem % j.nstrip, bandi = rem / j.nstrip;
    const int x0 = strip * kMetCols, oy0 = bandi * j.band, oy1 = min(oy0 + j.band, j.Ho);
    const int nrows = oy1 - oy0 + kWin - 1;   // input rows oy0 .. oy1 + 9 of the cropped grid
    const int t = threadIdx.x, col = x0 + t;
    const bool in_col = col < j.Wc;
    // squared error: every cropped pixel is counted by exactly one CTA
    const int own_x1 = strip == j.nstrip - 1 ? j.Wc : x0 + kMetCols;
    const int own_y1 = bandi == j.nband - 1 ? j.Hc : oy1;
    const bool own_col = col < own_x1;
    const bool out_col = t < kMetCols && col < j.Wo;
    const size_t plane = size_t(j.H) * j.W;
    const float* pa = j.pred + size_t(f) * 3 * plane + size_t(j.crop) * j.W + j.crop + min(col, j.Wc - 1);
    const float* pb = j.tgt + size_t(f) * 3 * plane + size_t(j.crop) * j.W + j.crop + min(col, j.Wc - 1);
    float ra[6], rb[6];
    auto fetch = [&](int row, float (&v)[6]) {   // row of the cropped grid
        const size_t o = size_t(row) * j.W;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            v[c] = __ldg(pa + c * plane + o);
            v[3 + c] = __ldg(pb + c * plane + o);
        }
    };
    fetch(oy0, ra);
    double ring[kWin][5];
    double ssim_sum = 0.0, sq_sum = 0.0;
    bool finite = true;
    for (int i0 = 0; i0 < nrows; i0 += kWin) {
#pragma unroll
        for (int ph = 0; ph < kWin; ++ph) {
            const int i = i0 + ph;
            if (i >= nrows) break;
#pragma unroll
            for (int k = 0; k < 6; ++k) rb[k] = ra[k];
            if (i + 1 < nrows) fetch(oy0 + i + 1, ra);
            double ya = 0.0, yb = 0.0;
            if (in_col) {
#pragma unroll
                for (int k = 0; k < 6; ++k) finite &= isfinite(rb[k]);
                ya = luma(clamp01(rb[0]), clamp01(rb[1]), clamp01(rb[2]));
                yb = luma(rb[3], rb[4], rb[5]);
                if (own_col && oy0 + i < own_y1) {
                    const double d = __dsub_rn(ya, yb);
                    sq_sum = __fma_rn(d, d, sq_sum);
                }
            }
            s_y[i & 1][t] = make_double2(ya, yb);
            __syncthreads();
            if (out_col) {
                double h[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
#pragma unroll
                for (int k = 0; k < kWin; ++k) {
                    const double2 v = s_y[i & 1][t + k];
                    const double w = j.g[k];
                    h[0] = __fma_rn(w, v.x, h[0]);
                    h[1] = __fma_rn(w, v.y, h[1]);
                    h[2] = __fma_rn(w, __dmul_rn(v.x, v.x), h[2]);
                    h[3] = __fma_rn(w, __dmul_rn(v.y, v.y), h[3]);
                    h[4] = __fma_rn(w, __dmul_rn(v.x, v.y), h[4]);
                }
#pragma unroll
                for (int q = 0; q < 5; ++q) ring[ph][q] = h[q];
                if (i >= kWin - 1) {   // window row oy0 + i - 10: ring rows i-10 .. i
                    double m[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
#pragma unroll
                    for (int k = 0; k < kWin; ++k) {
                        const int s = (ph + 1 + k) % kWin;   // slot of input row i - 10 + k
#pragma unroll
                        for (int q = 0; q < 5; ++q) m[q] = __fma_rn(j.g[k], ring[s][q], m[q]);
                    }
                    const double mab = __dmul_rn(m[0], m[1]);
                    const double maa = __dmul_rn(m[0], m[0]), mbb = __dmul_rn(m[1], m[1]);
                    const double va = __dsub_rn(m[2], maa), vb = __dsub_rn(m[3], mbb), cov = __dsub_rn(m[4], mab);
                    const double C1 = 0.01 * 0.01, C2 = 0.03 * 0.03;
                    const double num = __dmul_rn(__dadd_rn(__dmul_rn(2.0, mab), C1), __dadd_rn(__dmul_rn(2.0, cov), C2));
                    const double den = __dmul_rn(__dadd_rn(__dadd_rn(maa, mbb), C1), __dadd_rn(__dadd_rn(va, vb), C2));
                    ssim_sum = __dadd_rn(ssim_sum, __ddiv_rn(num, den));
                }
            }
        }
    }
    if (!finite) j.bad[f] = 1;
    // CTA reduction in a fixed order
    __shared__ double s_red[2][kMetThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ssim_sum += __shfl_down_sync(0xffffffffu, ssim_sum, o);
        sq_sum += __shfl_down_sync(0xffffffffu, sq_sum, o);
    }
    if ((t & 31) == 0) {
        s_red[0][t >> 5] = ssim_sum;
        s_red[1][t >> 5] = sq_sum;
    }
    __syncthreads();
    if (t == 0) {
        double a = 0.0, b = 0.0;
#pragma unroll
        for (int w = 0; w < kMetThreads / 32; ++w) {
            a += s_red[0][w];
            b += s_red[1][w];
        }
        j.partial[2 * size_t(blockIdx.x)] = a;
        j.partial[2 * size_t(blockIdx.x) + 1] = b;
    }
}

// Finite check of the cropped-away border (the window kernel reads only the crop), so that a
// non-finite value anywhere in either image is reported, as distortion() checks whole images.
__global__ void k_metric_border(const float* __restrict__ pred, const float* __restrict__ tgt, int n, int H, int W,
                                int crop, int* bad) {
    const long long side = (long long)(H - 2 * crop) * 2 * crop;   // left and right columns
    const long long per = 2LL * crop * W + side;                     // border pixels per frame
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < per * n; i += (long long)gridDim.x * blockDim.x) {
        const int f = int(i / per);
        const long long p = i % per;
        int y, x;
        if (p < 2LL * crop * W) {
            const int r = int(p / W);
            y = r < crop ? r : H - 2 * crop + r;
            x = int(p % W);
        } else {
            const long long q = p - 2LL * crop * W;
            y = crop + int(q / (2 * crop));
            const int c = int(q % (2 * crop));
            x = c < crop ? c : W - 2 * crop + c;
        }
        const size_t plane = size_t(H) * W, o = size_t(f) * 3 * plane + size_t(y) * W + x;
        bool ok = true;
#pragma unroll
        for (int c = 0; c < 3; ++c) ok &= isfinite(pred[o + c * plane]) && isfinite(tgt[o + c * plane]);
        if (!ok) bad[f] = 1;
    }
}

// Per-frame sums of the CTA partials, in a fixed order.
__global__ void k_metric_reduce(const double* __restrict__ partial, int per_frame, double* __restrict__ sums) {
    __shared__ double s[2][256];
    const int f = blockIdx.x, t = threadIdx.x;
    double a = 0.0, b = 0.0;
    for (int i = t; i < per_frame; i += 256) {
        a += partial[2 * (size_t(f) * per_frame + i)];
        b += partial[2 * (size_t(f) * per_frame + i) + 1];
    }
    s[0][t] = a;
    s[1][t] = b;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (t < o) {
            s[0][t] += s[0][t + o];
            s[1][t] += s[1][t + o];
        }
        __syncthreads();
    }
    if (t == 0) {
        sums[2 * f] = s[0][0];
        sums[2 * f + 1] = s[1][0];
    }
}

struct ScopedDevice {
    int prev = -1;
    explicit ScopedDevice(int dev) {
        AEISU_CUDA(cudaGetDevice(&prev));
        if (prev != dev) AEISU_CUDA(cudaSetDevice(dev));
    }
    ~ScopedDevice() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
    }
};

// Stream-ordered device allocation released on scope exit (on the same stream).
struct StreamBuf {
    void* p = nullptr;
    cudaStream_t s;
    StreamBuf(size_t bytes, cudaStream_t st) : s(st) { AEISU_CUDA(cudaMallocAsync(&p, bytes, st)); }
    ~StreamBuf() {
        if (p) cudaFreeAsync(p, s);
    }
};

}  // namespace

int metric_launches_per_call(int crop) { return crop > 0 ? 3 : 2; }

void distortion(const float* pred, const float* tgt, int n, int h, int w, int crop, bool host_io, int device,
                double* out, cudaStream_t stream) {
    require(out != nullptr, "output pointer is null");
    require(pred != nullptr && tgt != nullptr, "image pointer is null");
    require(n >= 1 && h >= 1 && w >= 1, "Prediction and target must be same-size CHW RGB");
    require(crop >= 0 && std::min(h, w) >= kWin + crop * 2,
            "Images are too small for the border crop and 11x11 SSIM window");
    ScopedDevice guard(device);
    MetricJob j{};
    j.H = h;
    j.W = w;
    j.crop = crop;
    j.Hc = h - 2 * crop;
    j.Wc = w - 2 * crop;
    j.Ho = j.Hc - (kWin - 1);
    j.Wo = j.Wc - (kWin - 1);
    j.nstrip = (j.Wo + kMetCols - 1) / kMetCols;
    // bands: one frame alone fills the SMs two CTAs deep, 64..256 rows per band (10 halo rows
    // each); the split depends on the frame size only, so a pair scores the same in any batch
    int sms = 148;
    AEISU_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    const long long rows = (long long)j.nstrip * j.Ho;
    const long long want = (rows + 2LL * sms - 1) / (2LL * sms);
    j.band = int(std::min<long long>(std::min<long long>(std::max<long long>(want, 64), 256), j.Ho));
    j.nband = (j.Ho + j.band - 1) / j.band;
    {   // torch: coordinate = arange(11) - 5; exp(-c^2 / (2 * 1.5^2)); / sum
        double s = 0.0;
        for (int k = 0; k < kWin; ++k) {
            const double c = double(k) - 5.0;
            j.g[k] = std::exp(-(c * c) / (2.0 * 1.5 * 1.5));
            s += j.g[k];
        }
        for (int k = 0; k < kWin; ++k) j.g[k] /= s;
    }
    const size_t frame = size_t(3) * h * w, bytes = frame * n * sizeof(float);
    const long long items = (long long)n * j.nstrip * j.nband;
    require(items < (1LL << 31), "batch too large");
    std::unique_ptr<StreamBuf> dpred, dtgt;
    if (host_io) {
        dpred = std::make_unique<StreamBuf>(bytes, stream);
        dtgt = std::make_unique<StreamBuf>(bytes, stream);
        AEISU_CUDA(cudaMemcpyAsync(dpred->p, pred, bytes, cudaMemcpyHostToDevice, stream));
        AEISU_CUDA(cudaMemcpyAsync(dtgt->p, tgt, bytes, cudaMemcpyHostToDevice, stream));
        j.pred = static_cast<const float*>(dpred->p);
        j.tgt = static_cast<const float*>(dtgt->p);
    } else {
        j.pred = pred;
        j.tgt = tgt;
    }
    const size_t ws_bytes = size_t(items) * 2 * sizeof(double) + size_t(n) * 2 * sizeof(double) + size_t(n) * sizeof(int);
    StreamBuf ws(ws_bytes, stream);
    j.partial = static_cast<double*>(ws.p);
    double* sums = j.partial + size_t(items) * 2;
    j.bad = reinterpret_cast<int*>(sums + size_t(n) * 2);
    AEISU_CUDA(cudaMemsetAsync(j.bad, 0, size_t(n) * sizeof(int), stream));
    k_metric_ssim<<<unsigned(items), kMetThreads, 0, stream>>>(j);
    AEISU_CUDA(cudaGetLastError());
    if (crop > 0) {
        const long long per = 2LL * crop * w + (long long)(h - 2 * crop) * 2 * crop;
        const int blocks = int(std::min<long long>((per * n + 255) / 256, 4LL * sms));
        k_metric_border<<<blocks, 256, 0, stream>>>(j.pred, j.tgt, n, h, w, crop, j.bad);
        AEISU_CUDA(cudaGetLastError());
    }
    k_metric_reduce<<<n, 256, 0, stream>>>(j.partial, j.nstrip * j.nband, sums);
    AEISU_CUDA(cudaGetLastError());
    std::vector<double> hs(size_t(n) * 2);
    std::vector<int> hb(n);
    AEISU_CUDA(cudaMemcpyAsync(hs.data(), sums, hs.size() * sizeof(double), cudaMemcpyDeviceToHost, stream));
    AEISU_CUDA(cudaMemcpyAsync(hb.data(), j.bad, hb.size() * sizeof(int), cudaMemcpyDeviceToHost, stream));
    AEISU_CUDA(cudaStreamSynchronize(stream));
    bool any_bad = false;
    const double nan = std::numeric_limits<double>::quiet_NaN();
    for (int f = 0; f < n; ++f) {
        double* o = out + 3 * size_t(f);
        if (hb[f]) {
            any_bad = true;
            o[0] = o[1] = o[2] = nan;
            continue;
        }
        const double mse = hs[2 * f + 1] / (double(j.Hc) * j.Wc);
        o[0] = mse;
        o[1] = mse == 0.0 ? std::numeric_limits<double>::infinity() : -10.0 * std::log10(mse);
        o[2] = hs[2 * f] / (double(j.Ho) * j.Wo);
    }
    if (any_bad) fail(AEISU_ERR_NONFINITE, "Prediction and target must be finite");
}

}  // namespace aeisu
