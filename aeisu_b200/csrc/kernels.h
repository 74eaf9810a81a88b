// Device-side descriptors shared by all kernel families, and their host launchers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

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

// FP32 parity route (k_f32.cu).  Activations are float32 NHWC.
void launch_f32_controller(const SrcDesc& src, const RegionSet& rs, const float* stencil,
                           const F32Layer* layers, float* enc540, float* low_a, float* low_b,
                           float* dec540, float* refined, float* meta, cudaStream_t s, int* launches,
                           const StageMark& mark);
void launch_f32_head(const SrcDesc& src, const RegionSet& rs, const DstDesc& dst,
                     const float* meta, const float* base, const float* basis, int* nonfinite,
                     cudaStream_t s, int* launches);

}  // namespace aeisu
