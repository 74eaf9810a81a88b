// Device-side descriptors shared by all kernel families, and their host launchers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <utility>
#include <vector>

#include "../../include/aeisu.h"

namespace aeisu {

// Source frames.  Padded-grid coordinate p maps to source pixel clamp(p - pad, 0, dim-1):
// the replicate padding of aeisu/runtime.py:81-84 folded into the index.
struct SrcDesc {
    const void* ptr;
    int kind;          // 0: uint8 HWC (value/255, runtime.py:17-20)  1: float32 CHW
    int H, W;
    int pad_y, pad_x;
};

// Output frames.  Region-local LR pixel (y, x) of region (oy, ox) writes output pixels
// (2*(oy + y - pad_y) + i, 2*(ox + x - pad_x) + j), i, j in {0, 1}.
struct DstDesc {
    void* ptr;
    int kind;          // 0: uint8 HWC, clamp + floor(x*255+0.5) (runtime.py:23-27)  1: float32 CHW unclipped
    int OH, OW;
    int pad_y, pad_x;
};

// A batch of equally sized regions of the padded grid (whole frames for tile=0, crops for
// tile>0, runtime.py:86-99).  Activations of region r live at index r of every buffer.
struct RegionSet {
    const int4* regions;  // {frame, oy, ox, 0}: region origin on the padded grid
    const int4* cores;    // {cy0, cx0, cy1, cx1}: region-local LR rectangle the head writes
    int R, rh, rw;        // region count, region height/width (multiples of 4)
    int core_h, core_w;   // largest core rectangle in the set (launch bounds of the head)
};

struct F32Layer { const float* w; const float* b; float slope; };

// Called after each controller stage has been enqueued (stage 1..4: analysis+project,
// compress+core, expand, refine+tail) so the engine can record timing events.
struct StageMark {
    void (*fn)(void* ctx, int stage) = nullptr;
    void* ctx = nullptr;
    void operator()(int stage) const { if (fn) fn(ctx, stage); }
};

// FP32 parity route (k_f32.cu).  Activations are float32 NHWC.  Calibration outputs (device,
// or null): peaks[10] accumulates the running max |x| of the ten activations the mixed route
// quantises, in SPYR8 activation_scales order (unshuffled features, project_540, compress_270,
// the four bottleneck outputs, expand_270 before the skip add, refine input, refine_540);
// sums[448] the per-input-channel sums of the FP8 layers: compress_270 (128, unshuffle order
// c*4 + phase), bottleneck 0-3 and expand_270 (64 each).
void launch_f32_controller(const SrcDesc& src, const RegionSet& rs, const float* stencil,
                           const F32Layer* layers, float* enc540, float* low_a, float* low_b,
                           float* dec540, float* refined, float* meta, cudaStream_t s, int* launches,
                           const StageMark& mark, float* peaks = nullptr, double* sums = nullptr);
// Scalar epilogue parameters of a tensor-core convolution layer; its per-channel accumulator
// multipliers (FP8: s_in * w_scale; INT8: factor) and biases travel beside it as ChannelParams.
struct EpiParams {
    float slope;          // LeakyReLU negative slope
    float out_inv;        // FP8 / INT8 output quantisation: 1/s_out
    float out_deq;        // expand: dequantisation s_out
};

// The feature-analysis stencil (24 values, SPYR8 analysis_stencil order) and project_540's bias,
// passed by value to the project kernel so that they sit in the constant bank.
struct ProjParams {
    float st[24];
    float bias[32];
};

// refine_540's and metadata_head's biases (the tail's as the route adds it), passed by value to
// the refine kernel so that they sit in the constant bank.
struct RefineBiases {
    float refine[64];
    float tail[64];
};

// Per-channel epilogue multipliers and biases of a 1x1 layer (compress_270: 64 channels,
// expand_270: 128), passed by value so that they sit in the constant bank.
template <int C>
struct ChannelParams {
    float scale[C];
    float bias[C];
};

// Device images of the tensor-core routes' weights, already in the K-major operand layout
// of tc.cuh (chunk-major, 16 bytes per row per chunk), plus per-channel epilogue vectors.
struct TcWeights {
    ProjParams proj;               // host copy of stencil and project bias
    RefineBiases rbias;            // host copy of the refine and tail biases
    ChannelParams<64> compress_cp;   // host copies of the 1x1 layers' epilogue vectors
    ChannelParams<64> core_cp[4];    // and of the bottleneck layers' (both groups)
    ChannelParams<128> expand_cp;
    const uint8_t* project;        // [4 chunks][32][16 B] f16
    float slope;
    float inv_s1;                  // 1/activation_scales[1] (e4m3 and int8 routes; else 1)
    const uint8_t* compress;       // [K/epc][64][16 B], K order phase*32 + c
    EpiParams compress_ep;
    const uint8_t* core[4];        // 2 groups x [9*32/epc][32][16 B], K order tap*32 + c
    EpiParams core_ep[4];
    const uint8_t* expand;         // [64/epc][128][16 B], N order phase*32 + c
    EpiParams expand_ep;
    const uint8_t* refine;         // [36][64][16 B] f16, K order tap*32 + c
    const uint8_t* tail;           // [8][64][16 B] f16
    const float* refine_bias;
    const float* tail_bias;
    const uint8_t* head;           // 3 x [2][128][16 B] f16: basis hi, basis lo, base hi|lo
};

// Controller routes of the tensor-core kernels: f16 activations everywhere; e4m3 compress /
// core / expand (the SPYR8 mixed route); int8 codes held as f16 in compress / core / expand
// (the shader_precision_v1 route: f16 MMAs over the codes give its exact integer sums).
enum TcRoute : int { kRouteF16 = 0, kRouteE4M3 = 1, kRouteI8 = 2 };
inline int tc_route_of(int precision) {
    return precision == AEISU_PRECISION_MIXED ? kRouteE4M3 : precision == AEISU_PRECISION_INT8 ? kRouteI8 : kRouteF16;
}

// Reconstruction fused into the controller's last stage: refine_540 + metadata_head + head in
// one kernel that writes the output frames, so the coefficients never reach HBM.
struct FusedHead {
    const DstDesc* dst;
    const uint8_t* head_img;
    int* nonfinite;
};

// Tensor-core route (k_tc.cu).
// Buffers are chunk-planar: enc540 [R][ph][4][pw][16], encu [R][lh][K/epc][lw][16],
// low [R][lh][64/epc][lw][16], dec540 [R][ph][4][pw][16], meta [R][rh][2][rw][16].
// With `head`, the last stage writes the output frames instead of meta (unused, may be null).
void launch_tc_controller(int route, const SrcDesc& src, const RegionSet& rs, const TcWeights& w, void* enc540,
                          void* encu, void* low_a, void* low_b, void* dec540, void* meta, float* raw_meta,
                          int* err, cudaStream_t s, int* launches, const StageMark& mark,
                          const FusedHead* head = nullptr);
void launch_tc_head(const SrcDesc& src, const RegionSet& rs, const DstDesc& dst, const void* meta,
                    const uint8_t* head_img, int* nonfinite, int* err, cudaStream_t s, int* launches);

void launch_f32_head(const SrcDesc& src, const RegionSet& rs, const DstDesc& dst,
                     const float* meta, const float* base, const float* basis, int* nonfinite,
                     cudaStream_t s, int* launches);

// Encoded-Y MSE / PSNR / SSIM of n image pairs (aeisu/metrics.py:17-39), k_metrics.cu.
// out[3f .. 3f+2] = y_mse, y_psnr, y_ssim of frame f; waits for completion.
void distortion(const float* pred, const float* tgt, int n, int h, int w, int crop, bool host_io, int device,
                double* out, cudaStream_t stream);
int metric_launches_per_call(int crop);

// PNG files of n frames (k_png.cu): kind 0 uint8 HWC, kind 1 float32 CHW quantised as save_rgb.
uint64_t png_bound(int h, int w);

// Dense tcgen05 throughput (TFLOP/s, best of `repeats` timed launches) of M = 128, N = 256 MMAs
// of kind 0 (f16, K = 16) or 1 (e4m3, K = 32) on `device` (k_peak.cu).
double tensor_peak_tflops(int device, int kind, int ctas_per_sm, int mmas, int repeats);
void png_encode(const void* src, int kind, int n, int h, int w, bool host_io, int device, uint8_t* out,
                uint64_t capacity, uint64_t* sizes, cudaStream_t stream);
int png_launches_per_call();

// PNG ingress (k_pngdec.cu): the header facts of one file, checked as PIL checks them, and, when
// `idat` is given, where its zlib stream lies in `data` (the IDAT payloads, in order, as
// (offset, length) pairs).
struct PngFileInfo {
    int w, h, depth, color, interlace, npal;
    uint8_t palette[768];
    unsigned long long idat_bytes;
};
PngFileInfo png_parse(const uint8_t* data, size_t size, std::vector<std::pair<size_t, size_t>>* idat);
// AEISU_ERR_UNSUPPORTED unless 8-bit samples, colour type 0/2/3/4/6, no interlacing.
void png_check_supported(const PngFileInfo& info);
// n PNG files (host memory) of one size h x w -> n uint8 RGB frames h x w x 3 in `out` (host or
// device memory); waits for completion.
void png_decode(const uint8_t* data, const uint64_t* offsets, const uint64_t* sizes, int n, int h, int w,
                bool host_out, int device, uint8_t* out, cudaStream_t stream);

// reconstruct() of aeisu/reconstruction.py:29-83 on caller-given metadata, base and basis, FP32,
// and its backward (k_recon.cu).  Device pointers; both only enqueue on `stream`.
void reconstruct_f32(const float* src, const float* meta, const float* base, const float* basis, int n, int h,
                     int w, int trim, int device, float* out, cudaStream_t stream);
void reconstruct_backward_f32(const float* src, const float* meta, const float* basis, const float* grad, int n,
                              int h, int w, int trim, int stride, int phase, int device, float* gmeta,
                              float* gbase, float* gbasis, cudaStream_t stream);

}  // namespace aeisu
