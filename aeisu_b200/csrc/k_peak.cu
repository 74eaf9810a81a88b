// Dense tensor-core throughput of this GPU, measured with the same tcgen05 instructions the
// controller kernels issue: the roofline denominators for the FP16 and FP8-E4M3 stages
// (the E4M3 rate is not part of the measured peaks the benchmark receives, which come from a
// cuBLAS BF16 GEMM).
//
// Each CTA stages one A tile (128 rows) and one B tile (256 rows) of K = 32 bytes per row in
// shared memory (K-major, no swizzle: K = 16 f16 or K = 32 e4m3 elements), allocates 256 TMEM
// columns and has one thread issue `mmas` back-to-back M = 128, N = 256 MMAs into the same
// accumulator, then one commit and a bounded wait.  N = 256 is the shape whose operands the
// tensor core reads from shared memory at full rate; two CTAs per SM keep the pipe fed while
// one of them is in its prologue or epilogue.  Operands hold a hashed bit pattern of finite
// values, so that the datapath toggles as it does on real data.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.h"
#include "kernels.h"
#include "tc_dev.cuh"

namespace aeisu {
namespace {

using namespace tc;
using namespace tcd;

constexpr int kPeakN = 256;
constexpr int kPeakABytes = 128 * 32, kPeakBBytes = kPeakN * 32;

template <bool FP8>
__global__ void __launch_bounds__(128) k_mma_peak(int mmas, int* err) {
    __shared__ __align__(128) uint8_t s_a[kPeakABytes];
    __shared__ __align__(128) uint8_t s_b[kPeakBBytes];
    __shared__ uint32_t s_tmem;
    __shared__ alignas(8) uint64_t s_bar;
    // operands: a fixed hashed bit pattern, masked so that every element is finite (f16
    // exponent field below 31; e4m3 codes without the all-ones NaN pattern)
    const uint32_t mask = FP8 ? 0x77777777u : 0x3BFF3BFFu;
    for (int i = threadIdx.x; i < (kPeakABytes + kPeakBBytes) / 4; i += blockDim.x) {
        uint32_t h = (uint32_t(i) + 0x9E3779B9u * (blockIdx.x + 1)) * 0x85EBCA6Bu;
        h ^= h >> 13;
        uint32_t* p = i < kPeakABytes / 4 ? reinterpret_cast<uint32_t*>(s_a) + i
                                            : reinterpret_cast<uint32_t*>(s_b) + (i - kPeakABytes / 4);
        *p = h & mask;
    }
    fence_async_smem();
    cta_setup(&s_tmem, &s_bar, 1, kPeakN);
    const uint32_t tmem = s_tmem;
    uint32_t phase = 0;
    if (threadIdx.x == 0) {
        // rows 16 B apart, the two 16-byte K chunks LBO apart, 8-row core matrices 128 B apart
        const uint64_t a = sdesc(smem_addr(s_a), 128 * 16, 128);
        const uint64_t b = sdesc(smem_addr(s_b), kPeakN * 16, 128);
        constexpr uint32_t idesc = idesc_m128(kPeakN);
        for (int i = 0; i < mmas; ++i) {
            if (FP8) mma_e4m3(tmem, a, b, idesc, i > 0);
            else mma_f16(tmem, a, b, idesc, i > 0);
        }
        commit(&s_bar);
    }
    mma_wait_all(&s_bar, phase, err);
    cta_teardown(tmem, kPeakN);
}

}  // namespace

double tensor_peak_tflops(int device, int kind, int ctas_per_sm, int mmas, int repeats) {
    require(kind == 0 || kind == 1, "kind must be 0 (f16) or 1 (e4m3)");
    require(ctas_per_sm >= 1 && ctas_per_sm <= 2, "ctas_per_sm must be 1 or 2 (256 TMEM columns each)");
    require(mmas >= 1 && mmas <= (1 << 20) && repeats >= 1 && repeats <= 1000, "mmas or repeats out of range");
    int prev = -1;
    AEISU_CUDA(cudaGetDevice(&prev));
    AEISU_CUDA(cudaSetDevice(device));
    int sms = 0;
    AEISU_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    cudaStream_t s = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int* err = nullptr;
    double best = 0.0;
    auto release = [&] {
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        if (err) cudaFree(err);
        if (s) cudaStreamDestroy(s);
        if (prev >= 0) cudaSetDevice(prev);
    };
    try {
        AEISU_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        AEISU_CUDA(cudaEventCreate(&e0));
        AEISU_CUDA(cudaEventCreate(&e1));
        AEISU_CUDA(cudaMalloc(&err, sizeof(int)));
        AEISU_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
        const unsigned grid = unsigned(sms * ctas_per_sm);
        auto kernel = kind == 1 ? k_mma_peak<true> : k_mma_peak<false>;
        for (int r = 0; r < repeats + 1; ++r) {   // the first launch warms up
            AEISU_CUDA(cudaEventRecord(e0, s));
            kernel<<<grid, 128, 0, s>>>(mmas, err);
            AEISU_CUDA(cudaGetLastError());
            AEISU_CUDA(cudaEventRecord(e1, s));
            AEISU_CUDA(cudaStreamSynchronize(s));
            float ms = 0.f;
            AEISU_CUDA(cudaEventElapsedTime(&ms, e0, e1));
            // 2 x M x N x K flops per MMA; K = 16 f16 or 32 e4m3 elements (32 bytes per row)
            const double flops = 2.0 * 128 * kPeakN * (kind == 1 ? 32 : 16) * double(mmas) * grid;
            if (r > 0) best = std::max(best, flops / (ms * 1e-3) / 1e12);
        }
        int flag = 0;
        AEISU_CUDA(cudaMemcpy(&flag, err, sizeof(int), cudaMemcpyDeviceToHost));
        require(flag == 0, "tensor peak kernel: a pipeline wait expired", AEISU_ERR_CUDA);
    } catch (...) {
        release();
        throw;
    }
    release();
    return best;
}

}  // namespace aeisu
