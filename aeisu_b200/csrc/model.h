// Host-side model: the deployed AEISU parameters in one precision-neutral form, plus
// the loaders for the two checkpoint formats the reference ships.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/aeisu.h"

namespace aeisu {

// Controller layers in execution order (aeisu/model.py:473-492).  The four grouped
// bottleneck layers hold both branches: weight [64, 32, 3, 3] = cat(a_i, b_i), groups=2,
// as the SPYR8 artifact stores them (optimized/native/src/neural/srcpyr/SrcPyrModel.cpp:441-449).
enum Layer : int {
    kProject = 0, kCompress, kCore0, kCore1, kCore2, kCore3, kExpand, kRefine, kTail, kLayerCount
};

struct LayerSpec { int cout, cin_per_group, k, groups; const char* spyr_name; };
extern const LayerSpec kLayerSpecs[kLayerCount];

struct LayerWeights {
    std::vector<float> w;          // OIHW float32 (FP32 master, or FP16 upcast from SPYR8)
    std::vector<float> bias;       // [cout]
    std::vector<float> bias_fp8;   // bias the FP8 epilogue adds (SPYR8 `.bias_fp8`; else = bias)
    std::vector<float> slope;      // LeakyReLU negative slope per output channel (tail: 1 = linear)
    std::vector<uint16_t> w_fp16;  // OIHW IEEE half bits
    std::vector<uint8_t> w_fp8;    // OIHW E4M3 codes (SPYR8 only)
    std::vector<float> w_scale;    // per-output-channel FP8 weight scale (SPYR8 only)
    std::vector<float> factor;     // per-output-channel INT8 accumulator multiplier (INT8 artifact only;
                                   // w / w_fp16 then hold the int8 codes)
};

struct HostModel {
    // analysis stencil: rgbBasis[9] (row-major), rgbMix[3], dxRows[3], dyCols[3], diag45[3],
    // diag135[3] (SrcPyrArchitecture.h:42-51 LearnedAnalysis4Dir order)
    float stencil[24];
    float base[25 * 4];        // [tap][phase]     (model.py:588-589)
    float basis[25 * 16 * 4];  // [tap][k][phase]  projected (reconstruction.py:8-12)
    LayerWeights layers[kLayerCount];
    float act_scales[10] = {};  // SPYR8 activation scales (Appendix of the artifact contract)
    // Power-of-two factor the mixed route applies to act_scales (1 = the artifact's own
    // quantisation points, as the reference's mixed route runs them)
    float fp8_headroom = 1.0f;
    bool has_fp8 = false;
    bool has_int8 = false;      // INT8 artifact: compress/core/expand as int8 codes and factors
    std::string format;         // "folded", "spyr8" or "shader_int8"
    std::string checksum_hex;   // SPYR8 SHA-256
    std::string architecture;
};

// Folded checkpoint: FoldedAEISU.state_dict() tensors concatenated in order.
HostModel load_folded(const float* values, size_t count, float basis_l1_scale);

// SPYR8 v1 artifact bytes (parsing and validation of SrcPyrModel.cpp:243-470, restated).
HostModel load_spyr8(const uint8_t* data, size_t bytes);

// INT8/FP16 artifact arrays (shader_precision_v1), validated.
HostModel load_int8(const aeisu_int8_artifact& a);

// IEEE binary16 helpers (round to nearest even).
uint16_t f32_to_f16_bits(float f);
float f16_bits_to_f32(uint16_t h);
// OCP FP8 E4M3 (finite-only "fn" variant) decode.
float e4m3_to_f32(uint8_t code);

}  // namespace aeisu
