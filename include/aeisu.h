/*
 * aeisu.h — C ABI of the B200 (sm_100a) AEISU 2x inference runtime.
 *
 * One handle = one model resident on one GPU (weights, packed operand layouts,
 * workspace, CUDA stream).  Calls on one handle are not thread-safe; use one handle
 * per host thread: aeisu_open_sibling gives another handle that shares the weights.  The caller owns every I/O
 * buffer; the library owns weights and workspace.  Every entry point returns an
 * aeisu_status (never throws); aeisu_last_error() gives the calling thread's last
 * message.
 *
 * Reference interfaces replaced (paths relative to the AELabs42/AEISU checkout):
 *   aess::srcpyr::ModelArtifact::Load      optimized/native/src/neural/srcpyr/SrcPyrModel.cpp:243-470
 *   aess::srcpyr::CudaRuntime (ctor, Configure, Process, StartupReport, PersistentDeviceBytes)
 *                                          optimized/native/src/neural/srcpyr/SrcPyrCudaRuntime.h:29-96
 *   aeisu.runtime.load_model               aeisu/runtime.py:45-56
 *   aeisu.runtime.upscale                  aeisu/runtime.py:70-103
 *   FoldedAEISU.forward / predict_coefficients   aeisu/model.py:494-551
 *   aeisu.metrics.distortion               aeisu/metrics.py:17-39 (evaluate.py:41)
 *   aeisu.runtime.save_rgb (PNG egress)    aeisu/runtime.py:23-27 (infer.py, evaluate.py:48)
 *   aeisu.reconstruction.reconstruct (forward and its autograd backward)
 *                                          aeisu/reconstruction.py:29-83 (train.py:99-103)
 * The Python binding that mirrors aeisu.runtime over this ABI is aeisu_b200/runtime.py.
 */
#ifndef AEISU_B200_H
#define AEISU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct aeisu_engine aeisu_t;

/* Status codes.  The reference raises std::runtime_error (native) or ValueError /
 * FloatingPointError (aeisu/runtime.py:77-80, 101-102); these are their C forms. */
typedef enum aeisu_status {
    AEISU_OK = 0,
    AEISU_ERR_INVALID_ARG = 1,   /* ValueError: shape, tile, pointer, flag misuse      */
    AEISU_ERR_BAD_ARTIFACT = 2,  /* artifact parse / checksum / contract failure       */
    AEISU_ERR_CUDA = 3,          /* a CUDA runtime or driver call failed               */
    AEISU_ERR_NONFINITE = 4,     /* FloatingPointError: non-finite reconstruction      */
    AEISU_ERR_TIMEOUT = 5,       /* a bounded wait for GPU completion expired          */
    AEISU_ERR_UNSUPPORTED = 6,   /* precision/format combination not available         */
    AEISU_ERR_OOM = 7            /* device or host allocation failed                   */
} aeisu_status;

/* Arithmetic of the controller convolutions (the head always accumulates in FP32).
 * FP32  : every layer FP32 (the parity path; aeisu/model.py semantics).
 * FP16  : FP16 operands, FP32 accumulate (reference "Fp16" route).
 * MIXED : FP8-E4M3 compress/core/expand, FP16 project/refine/tail, as laid out by
 *         the SPYR8 artifact (reference "Mixed" route, SrcPyrCudaRuntime.cu:4131-4873).
 * INT8  : int8 compress/core/expand, FP16 project/refine/tail, as the shader_precision_v1
 *         artifact lays out (conventional-CUDA route, optimized/shader/runtime.py:173-221):
 *         int8 activation codes at the artifact's scales, per-channel factors and biases; the
 *         codes run as f16 on the tensor cores, whose FP32 sums of them are the exact integer
 *         dot products.  Only models opened with aeisu_open_int8 have it. */
typedef enum aeisu_precision {
    AEISU_PRECISION_FP32 = 0,
    AEISU_PRECISION_FP16 = 1,
    AEISU_PRECISION_MIXED = 2,
    AEISU_PRECISION_INT8 = 3
} aeisu_precision;

/* Flags for the I/O calls. */
#define AEISU_IO_HOST   0u   /* src/dst are host pointers (pinned for full PCIe speed); the
                                call copies, runs and waits (bounded by the handle timeout) */
#define AEISU_IO_DEVICE 1u   /* src/dst are device pointers on the handle's GPU; the call only
                                enqueues on `stream` (or the handle's stream when NULL, which
                                is not ordered with the legacy default stream: pass
                                cudaStreamLegacy to run after work queued there)              */

/* Number of float values in a folded checkpoint (aeisu/model.py:554-583, 34 tensors,
 * tests/test_reference.py:69). */
#define AEISU_FOLDED_VALUES 115996

/* Open a model from a SPYR8 v1 artifact file (adaptive_fp8.bin layout).
 * Replaces ModelArtifact::Load + CudaRuntime(modelPath): same header, descriptor,
 * SHA-256 (checksum field zeroed) and zero-DC/L1 basis contract checks. */
int aeisu_open_spyr8(const char* path, int precision, int device, aeisu_t** out);

/* Parse and validate a SPYR8 artifact image on the host only (no GPU needed): header,
 * descriptors, SHA-256, tensor contract.  On success writes the 64-hex-digit checksum and
 * a NUL to checksum_hex (at least 65 bytes) when it is not NULL. */
int aeisu_validate_spyr8(const void* data, size_t bytes, char* checksum_hex);

/* Same as aeisu_open_spyr8, from an artifact image already in host memory. */
int aeisu_open_spyr8_memory(const void* data, size_t bytes, int precision, int device,
                            aeisu_t** out);

/* aeisu_open_spyr8_memory with the mixed route's FP8 activation scales multiplied by
 * `activation_headroom`, a power of two in [1, 64] (1 gives exactly aeisu_open_spyr8_memory:
 * the artifact's own scales, as the reference applies them, SrcPyrCudaRuntime.cu:4427-4451,
 * 4587-4601).  E4M3 is a floating-point format, so a power-of-two factor h leaves the rounding
 * of every activation below the artifact's saturation limit unchanged and only keeps values in
 * [448 s, 448 h s) from saturating: content beyond the artifact's calibration range (the
 * reference calibrated on natural images) then keeps its magnitude, at the cost of h times
 * coarser rounding of values below 2^-6 s.  Only the mixed route reads it. */
int aeisu_open_spyr8_headroom(const void* data, size_t bytes, int precision, int device,
                              float activation_headroom, aeisu_t** out);

/* Open a model from folded FP32 weights: the 34 tensors of FoldedAEISU.state_dict()
 * concatenated in that order (AEISU_FOLDED_VALUES floats), plus basis_l1_scale.
 * Replaces load_model(path) for folded .pt checkpoints (aeisu/runtime.py:45-56);
 * the Python binding reads the .pt and passes its tensors here.  Precision FP32 or
 * FP16 (MIXED needs the FP8 scales of a SPYR8 artifact). */
int aeisu_open_folded(const float* values, size_t count, float basis_l1_scale,
                      int precision, int device, aeisu_t** out);

/* The shader_precision_v1 INT8/FP16 artifact (optimized/shader/weights/aeisu_int8_fp16.pt as
 * MixedRuntime reads it, optimized/shader/runtime.py:37-59) as plain host arrays; the Python
 * binding (aeisu_b200.load_model) unpacks the .pt and checks its format and precision policy
 * as runtime.py:41-43 does.  Weights are OIHW; the four bottleneck tensors hold both branches
 * ([64][32][3][3], groups 2); half weights are IEEE binary16 bits.  Replaces
 * MixedRuntime.__init__ (runtime.py:37-59). */
typedef struct aeisu_int8_artifact {
    const float* analysis;           /* [24] analysis_parameters (rgb basis, mix, dx, dy, d45, d135) */
    const float* base;               /* [25][4] */
    const float* bank;               /* [25][16][4] projected basis */
    const uint16_t* project_w;       /* [32][32]          half_weights["project"] */
    const uint16_t* refine_w;        /* [64][32][3][3]    half_weights["refine"] */
    const uint16_t* tail_w;          /* [64][64]          half_weights["tail"] */
    const float* project_b;          /* [32]  half_biases */
    const float* refine_b;           /* [64] */
    const float* tail_b;             /* [64] */
    const int8_t* int8_w[6];         /* compress [64][128], bottleneck0..3 [64][32][3][3], expand [128][64] */
    const float* int8_factor[6];     /* per output channel: accumulator multiplier */
    const float* int8_bias[6];       /* per output channel */
    const float* activation_scales;  /* [10] */
} aeisu_int8_artifact;

/* Open a model from the INT8/FP16 artifact on GPU `device`; its only precision is
 * AEISU_PRECISION_INT8.  AEISU_ERR_BAD_ARTIFACT for a missing array, a non-finite value, a
 * non-positive scale or a weight code outside [-127, 127]. */
int aeisu_open_int8(const aeisu_int8_artifact* artifact, int device, aeisu_t** out);

/* A sibling of `handle`, like CudaRuntime::CreateSibling (SrcPyrCudaRuntime.cu:5392-5402): the
 * same model, precision and GPU, sharing the handle's device weights (one copy per model and
 * device, released with the last handle that shares it), with its own CUDA stream, workspace,
 * status flags and timings.  Unlike the reference's siblings, which share one engine and stream,
 * siblings may run on different host threads at the same time; each handle is still used by one
 * thread at a time.  Closing the original handle first is allowed. */
int aeisu_open_sibling(aeisu_t* handle, aeisu_t** out);

void aeisu_close(aeisu_t* handle);

/* uint8 RGB in, uint8 RGB out: n frames of h x w x 3 (HWC, row-major, contiguous)
 * -> n frames of 2h x 2w x 3.  Semantics of upscale(model, read_rgb(x), tile) followed
 * by save_rgb's clamp and floor(x*255+0.5) (aeisu/runtime.py:17-27, 70-103):
 * replicate align-32 + 16 halo padding, tile == 0 full frame, tile > 0 (multiple of
 * 32) cores on the padded grid with 32-LR-pixel halos.  Returns AEISU_ERR_NONFINITE
 * if any reconstruction value is not finite (host I/O; with device I/O the flag is
 * reported by aeisu_synchronize). */
int aeisu_upscale_u8(aeisu_t* handle, const uint8_t* src, int n, int h, int w, int tile,
                     uint8_t* dst, unsigned flags, void* stream);

/* One row band of a single frame: aeisu_upscale_u8 with n = 1 and tile = 0, restricted to band
 * `band` of `bands`.  The padded grid's rows are split into `bands` equal bands (a multiple of
 * 32 rows each, the last one shorter); a band is computed on its rows plus 32 halo rows above
 * and below (clipped to the grid), over the full width, like one tile of the reference's tiled
 * path (aeisu/runtime.py:89-99).  The controller's receptive field is smaller than the halo,
 * so the band's output rows equal those of the whole-frame call bit for bit.  src and dst are
 * the whole frame (h x w x 3 in, 2h x 2w x 3 out); only the band's output rows are written,
 * and with host I/O only the source rows the band reads are copied.  No reference counterpart:
 * this is the single-huge-frame split across GPUs (one band per GPU, no data exchange). */
int aeisu_upscale_u8_band(aeisu_t* handle, const uint8_t* src, int h, int w, int band, int bands,
                          uint8_t* dst, unsigned flags, void* stream);

/* Allocation-free variant of aeisu_upscale_u8 with device I/O and tile = 0 (no counterpart
 * in the reference).  For hosts that must not allocate GPU memory when they submit a frame
 * (a presentation loop that cannot stall on cudaMalloc, a process with a fixed memory budget,
 * a caller that owns every buffer): all intermediate tensors live in one static device array
 * of 64 MiB that every GPU loading the library holds until exit.  src/dst are device
 * pointers (n frames of h x w x 3 uint8 in, 2h x 2w x 3 out); work is enqueued on `stream`
 * (NULL: the handle's stream) and the call returns without waiting.  The scratch a frame
 * needs is about 80 bytes per padded input pixel on the mixed route, 96 on FP16 and INT8 and
 * 224 on FP32, so the largest frames are about 0.83, 0.69 and 0.29 Mpixel of padded input
 * (the padded grid rounds h and w up to a multiple of 32 and adds 32): 960x540 fits the
 * mixed, FP16 and INT8 routes, 640x360 the FP32 route.  Larger frames are rejected with
 * AEISU_ERR_INVALID_ARG; batches run in as many passes of whole frames as the array needs.
 * The array is shared and keeps the previous call's contents: calls whose GPU work overlaps
 * in time race and must be serialised.  The first call on a device looks up the array's
 * address, and the first call on a device and shape may set kernel attributes and add entries
 * to small host-side caches (kernel attributes, TMA tensor maps of the scratch array); make
 * that first call before any stream capture.
 * The cached address is not refreshed after cudaDeviceReset: a handle and this entry point
 * must not outlive a reset of their device.  Non-finite outputs are reported by
 * aeisu_synchronize. */
int aeisu_upscale_u8_noalloc(aeisu_t* handle, const uint8_t* src, int n, int h, int w,
                             uint8_t* dst, void* stream);

/* Float parity path: n frames of float32 CHW (3 x h x w, values as read_rgb gives) ->
 * UNCLIPPED float32 CHW 3 x 2h x 2w (clip and the finite check are the caller's, as in
 * aeisu/runtime.py:100-103). */
int aeisu_upscale_f32(aeisu_t* handle, const float* src, int n, int h, int w, int tile,
                      float* dst, unsigned flags, void* stream);

/* FoldedAEISU.forward on an already padded NCHW float32 batch (h, w multiples of 4):
 * unclipped [n,3,2h,2w] (aeisu/model.py:546-551). */
int aeisu_forward_f32(aeisu_t* handle, const float* src, int n, int h, int w, float* dst,
                      unsigned flags, void* stream);

/* FoldedAEISU.predict_coefficients on an NCHW float32 batch (h, w multiples of 4):
 * metadata as float32 NHWC [n, h/2, w/2, 64], channel = parity*16 + component
 * (aeisu/model.py:494-496; reconstruction.py:20-26).  Values are the raw head output
 * (before coefficient_clamp), in the handle's precision. */
int aeisu_predict_coefficients(aeisu_t* handle, const float* src, int n, int h, int w,
                               float* meta, unsigned flags, void* stream);

/* Calibration for the SPYR8 exporter: runs the FP32 controller of a handle opened with
 * AEISU_PRECISION_FP32 over n uint8 frames (h x w x 3, padded as aeisu_upscale_u8 with tile 0
 * pads them) and writes (host memory):
 *   peaks[10]  the largest |x| of the ten activations the mixed route quantises, in the order
 *              of the SPYR8 activation_scales tensor: unshuffled analysis features,
 *              project_540, compress_270, bottleneck 1-4, expand_270 before the skip add, the
 *              refine input, refine_540;
 *   means[448] (may be NULL) the mean of each input channel of the FP8 layers: compress_270
 *              (128, in its unshuffled order c*4 + phase), bottleneck 1-4 and expand_270 (64
 *              each), for the bias correction of their E4M3 weights.
 * The SPYR8 layout is SrcPyrModel.cpp:37-85; the reference's calibrator itself is not shipped.
 * Waits for completion.  AEISU_ERR_UNSUPPORTED for other precisions. */
int aeisu_activation_stats(aeisu_t* handle, const uint8_t* src, int n, int h, int w, unsigned flags,
                           float* peaks, float* means, void* stream);

/* Evaluation metrics, no model needed: distortion() of aeisu/metrics.py:17-39 (called per image
 * pair by evaluate.py:41) on n pairs of float32 CHW images (3 x h x w each: the prediction as
 * upscale returns it, the target as read_rgb gives it), computed in FP64 on GPU `device`:
 * prediction clamped to [0, 1], both cropped by `crop` pixels per side, BT.601 encoded luma,
 * out[3i + 0] = y_mse, out[3i + 1] = y_psnr (+inf when the MSE is 0), out[3i + 2] = y_ssim
 * (mean over the valid 11x11 Gaussian windows, sigma 1.5).  Results agree with the reference
 * to FP64 rounding (separable window sums; the reference's own tolerance for these figures is
 * 2e-10).  flags: AEISU_IO_HOST or AEISU_IO_DEVICE for both images; `out` is host memory and
 * the call waits.  AEISU_ERR_INVALID_ARG when min(h, w) < 11 + 2 crop or crop < 0;
 * AEISU_ERR_NONFINITE when any value of either image is not finite (that pair's outputs are
 * NaN, the others are still written). */
int aeisu_distortion(const float* prediction, const float* target, int n, int h, int w, int crop,
                     unsigned flags, int device, double* out, void* stream);

/* PNG egress on the GPU: the files save_rgb writes (aeisu/runtime.py:23-27), for n frames at
 * once.  kind AEISU_PNG_U8: frames are uint8 h x w x 3 (HWC, as aeisu_upscale_u8 writes them);
 * kind AEISU_PNG_F32: frames are float32 3 x h x w (CHW, as aeisu_upscale_f32 writes them),
 * quantised as save_rgb does (clamp to [0, 1], floor(x * 255 + 0.5)).  The files are 8-bit RGB,
 * non-interlaced, adaptively filtered per row; their pixels decode to exactly save_rgb's, the
 * compressed stream is the encoder's own (one dynamic Huffman block per 60 KiB segment, with
 * greedy single-candidate LZ77 matches, not zlib's chained lazy matching), so the file bytes
 * and sizes differ from PIL's.  flags: where the frames are,
 * AEISU_IO_HOST or AEISU_IO_DEVICE (on GPU `device`); `out` may be host or device memory.
 * The n files are written back to back into `out` (capacity bytes;
 * n * aeisu_png_bound(h, w) always suffices) and sizes[i]
 * (host) receives each file's length; AEISU_ERR_INVALID_ARG if they do not fit (sizes[] is
 * filled first).  Widths above 32768 are rejected.  The call waits for completion. */
#define AEISU_PNG_U8  0
#define AEISU_PNG_F32 1
int aeisu_png_encode(const void* frames, int kind, int n, int h, int w, unsigned flags, int device,
                     uint8_t* out, uint64_t capacity, uint64_t* sizes, void* stream);

/* Largest PNG file aeisu_png_encode can produce for one h x w frame (0 for an empty size). */
uint64_t aeisu_png_bound(int h, int w);

/* PNG ingress, host side only: checks one PNG file in host memory as PIL's PngImagePlugin does
 * (signature, chunk layout, the CRC of every chunk before the image data, IHDR, PLTE) and
 * returns its size and colour type.  AEISU_ERR_UNSUPPORTED for
 * what aeisu_png_decode does not take (bit depths other than 8, interlaced files);
 * AEISU_ERR_INVALID_ARG for a broken file (PIL's PngImagePlugin raises for the same). */
int aeisu_png_info(const uint8_t* file, uint64_t bytes, int* h, int* w, int* color_type);

/* PNG ingress on the GPU: the decode of read_rgb (aeisu/runtime.py:17-20: PIL open, convert("RGB"),
 * uint8 HWC) for n PNG files at once.  The files lie back to back or anywhere in host memory
 * (file i at files + offsets[i], sizes[i] bytes) and must all be h x w; 8-bit samples of colour
 * type 0 (grey), 2 (RGB), 3 (palette), 4 (grey + alpha) or 6 (RGBA), not interlaced.  out
 * receives n frames of h x w x 3 uint8 RGB (HWC), in host or device memory on GPU `device`
 * (flags AEISU_IO_HOST / AEISU_IO_DEVICE); grey is replicated, palettes looked up and alpha
 * dropped, as convert("RGB") does, so the pixels equal PIL's.  The chunks are parsed and
 * CRC-checked on the host as PIL checks them (the chunks before the image data); on the GPU one
 * CTA per file: a warp inflates its zlib stream (deflate is sequential within a stream: the
 * parallelism is across files) while a second warp undoes the scanline filters of each group of
 * 32 rows already inflated, converts to RGB and checks the stream's Adler-32.  What PIL
 * tolerates is tolerated (image data past the image, a missing Adler-32 trailer, bad CRCs from
 * the first IDAT chunk on).  Waits for completion.  AEISU_ERR_INVALID_ARG for a broken or
 * differently sized file (the message names it), AEISU_ERR_UNSUPPORTED as for aeisu_png_info.  Keeps its device buffers between calls (per
 * device, grow-only; calls on one device take turns); like the no-allocation entry point's
 * cache, they do not survive cudaDeviceReset. */
int aeisu_png_decode(const uint8_t* files, const uint64_t* offsets, const uint64_t* sizes, int n, int h, int w,
                     unsigned flags, int device, uint8_t* out, void* stream);

/* reconstruct() of aeisu/reconstruction.py:29-83 as a standalone FP32 operator (the function
 * train.py:99-103 differentiates), no model handle needed.  All pointers are device memory on
 * GPU `device`, contiguous float32: source [n][3][h][w], metadata [n][64][h/2][w/2] (channel
 * parity * 16 + k, unclamped), base [25][4] (tap, phase), basis [25][16][4] (tap, component,
 * phase: project_basis's output).  trim as the reference's: 0, or an even HR border >= 4, so
 * the core is (h - trim) x (w - trim) LR pixels, read with replicate padding at trim 0 and the
 * real border otherwise.  out [n][3][2ch][2cw] (ch = h - trim, cw = w - trim) receives the
 * unclipped 2x core.  Enqueues on `stream` (NULL: the legacy default stream)
 * and returns.  AEISU_ERR_INVALID_ARG with the reference's messages for a bad trim, stride or
 * phase, an empty core, odd h or w. */
int aeisu_reconstruct_f32(const float* source, const float* metadata, const float* base, const float* basis,
                          int n, int h, int w, int trim, int device, float* out, void* stream);

/* Backward of aeisu_reconstruct_f32 with the reference's sampled global-filter gradients
 * (reconstruction.py:56-78): given grad_out [n][3][2ch][2cw], writes grad_metadata (same
 * layout as metadata; dense, through the coefficient clamp; zero outside the core) and, when
 * gradient_stride > 0, grad_base [25][4] and grad_basis [25][16][4]: over every core pixel at
 * stride 1, otherwise over the pixels with y % s == phase' / s and x % s == phase' % s (core
 * coordinates, phase' = phase mod s^2), each weighted s^2.  gradient_stride 0 leaves
 * grad_base and grad_basis untouched (they may be NULL): the reference gives them no
 * gradient.  Gradients with respect to the source are not computed.  The filter-gradient
 * sums are deterministic for a given GPU.  Takes a small stream-ordered workspace (6.8 KB per
 * SM-resident CTA) from a memory pool the library keeps per device, and enqueues on `stream`. */
int aeisu_reconstruct_backward_f32(const float* source, const float* metadata, const float* basis,
                                   const float* grad_out, int n, int h, int w, int trim, int gradient_stride,
                                   int phase, int device, float* grad_metadata, float* grad_base,
                                   float* grad_basis, void* stream);

/* Measurement helper with no counterpart in the reference: the dense tensor-core throughput of
 * GPU `device` for the instructions the controller kernels issue, as the roofline denominator
 * of their stages.  kind 0: tcgen05.mma kind::f16 (f16 operands, K = 16); kind 1: kind::f8f6f4
 * with E4M3 operands (K = 32).  Each of ctas_per_sm (1 or 2) CTAs per SM issues mmas_per_cta
 * back-to-back M = 128, N = 256 MMAs from one thread into one TMEM accumulator; *tflops
 * receives 2 * 128 * 256 * K * MMAs / time, the best of `repeats` launches timed with CUDA
 * events (one untimed launch first).  Waits for completion; allocates 4 bytes of device
 * memory for the kernel's error flag. */
int aeisu_tensor_peak(int device, int kind, int ctas_per_sm, int mmas_per_cta, int repeats, double* tflops);

/* Wait for all work enqueued on the handle's stream (or `stream`) for at most
 * timeout_ms; AEISU_ERR_TIMEOUT if it has not finished, AEISU_ERR_NONFINITE if a
 * reconstruction since the last call produced a non-finite value. */
int aeisu_synchronize(aeisu_t* handle, void* stream, double timeout_ms);

/* Per-stage device times of the last upscale call, in milliseconds (CUDA events;
 * replaces FrameTimings, NeuralRuntimeTypes.h:36-52). */
typedef struct aeisu_timings {
    float analysis_project_ms;   /* feature analysis + unshuffle + project_540          */
    float compress_core_ms;      /* compress_270 + 4 grouped bottleneck layers           */
    float expand_ms;             /* expand_270 + pixel shuffle + skip add                */
    float refine_tail_ms;        /* refine_540 + metadata_head                           */
    float reconstruction_ms;     /* fused reconstruction head                            */
    float total_ms;              /* first to last event, including host<->device copies */
    int   detailed;              /* 1 when the stage split was recorded                  */
} aeisu_timings;

int aeisu_timings_get(aeisu_t* handle, aeisu_timings* out);
int aeisu_set_detailed_timing(aeisu_t* handle, int enabled);

/* Implementation switch with no counterpart in the reference.  Tensor-core routes (FP16,
 * mixed, INT8): where the reconstruction head runs.  enabled = 0 (default): a separate head
 * kernel reads the clamped coefficients back from a workspace tensor (32 bytes per LR pixel), as
 * the reference's fused refine+tail kernel and ReconstructConstant pass them
 * (SrcPyrCudaRuntime.cu:4662-4666, 4831-4834).  enabled = 1: inside the controller's last kernel
 * (refine_540 + metadata_head + head), so the coefficients stay in shared memory and never reach
 * device memory and the workspace tensor is not allocated; refine_tail_ms then holds both stages
 * and reconstruction_ms is 0.  The output is the same bit for bit; on a B200 the fused kernel
 * measures slower (eight warps per SM against the two kernels' 16 and 18).  The FP32 route
 * always runs its separate head. */
int aeisu_set_fused_head(aeisu_t* handle, int enabled);

/* Bound, in milliseconds, on every host wait for GPU completion (default 60000). */
int aeisu_set_timeout(aeisu_t* handle, double timeout_ms);

/* Bound on the intermediate-tensor bytes one call allocates (default 6 GiB).  A batch of
 * regions (frames or tiles) that needs more is run in several passes of as many regions as
 * fit, at least one; the results are the same.  For hosts with a device memory budget. */
int aeisu_set_workspace_limit(aeisu_t* handle, uint64_t bytes);

/* Startup report (device, artifact hash, precision, kernel route), like
 * CudaRuntime::StartupReport (SrcPyrCudaRuntime.cu:3739-3783).  Valid until close. */
const char* aeisu_report(aeisu_t* handle);

/* Bytes of device memory the handle holds (weights, shared ones included, + workspace). */
uint64_t aeisu_device_bytes(aeisu_t* handle);

/* Number of kernels the library launched on this handle since it was opened. */
uint64_t aeisu_kernel_launches(aeisu_t* handle);

/* Message of the last failure on the calling thread ("" if none). */
const char* aeisu_last_error(void);

/* Library version string. */
const char* aeisu_version(void);

#ifdef __cplusplus
}
#endif
#endif /* AEISU_B200_H */
